#!/usr/bin/env python
"""Listener-step benchmark: frames/s of the streaming listener on B200.

Workload (per GPU): the d=1536 / 12-layer Gemma 4 audio
Conformer with weight-only int8 (per-output-channel fp16 scales) on every
Conformer linear and the FiLM adapter, `--sessions` concurrent sessions per
GPU under ragged arrivals (sessions of Geometric(1/300) length run back to back
in each lane, so sessions join and leave every step with differing cache
positions).  One step = one 80 ms tick for every live session:
pack (GPU slot policy) -> PCM log-mel -> Conformer -> soft tokens -> FiLM -> commit.

`value` is whole-job frames/s with inputs resident in HBM; `e2e` is the same
tick through the C ABI with host buffers (lb_step_host: H2D of rows, PCM and
FiLM queries, D2H of soft tokens and FiLM outputs inside the timed region).
Multi-GPU: one process per GPU (torchrun), sessions sharded by id, no
collective on the step; timings are the max over ranks.

Extra keys of the same line: `latency_e2e` (p50/p99 over 500 end-to-end ticks
at the benched N), `small_n` (weight-streaming regime, N in {1, 4, 16, 64}:
step time and achieved HBM GB/s against the step's algorithmic bytes),
`capacity_sweep` (end-to-end p50/p99 per N; `realtime_sessions_per_gpu` is the
largest N whose end-to-end p99 < 20 ms), and `config4` (
8192 sessions in total sharded by session id over the job's GPUs, 2000 steps).

`--impl reference` times the CPU port of the reference path (mel + Conformer +
FiLM in fp32 on all host cores; the port is pinned to goldens of the
reference's own classes, which cannot be installed as a package) on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "listener frames/sec (80 ms frames), whole job"
UNIT = "frames/s"


def load_package():
    name = "gemma4_omni_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = ROOT / "gemma-4-omni_b200"
    spec = importlib.util.spec_from_file_location(name, pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def wide_min_tokens() -> int:
    """Smallest token bucket whose int8 GEMMs read the fp16-widened codes (the
    library's default, or LB_WIDE_MIN_TOKENS as the library reads it)."""
    return max(0, int(os.environ.get("LB_WIDE_MIN_TOKENS", "128")))


def token_tile(O: int, m: int, sms: int = 148) -> int:
    """The GEMM's token tile for an [m x O] output (csrc/gemm_tc.cu gemm_token_tile)."""
    for cap in (32, 64, 128, 256):
        if m <= cap:
            return cap
    best, best_cost = 256, None
    for tn in (256, 240, 224, 208, 192, 176, 160, 144, 128):
        units = (O // 128) * -(-m // tn)
        cost = -(-units // sms) * (tn + 32)
        if best_cost is None or cost < best_cost:
            best, best_cost = tn, cost
    return best


def step_splits(O: int, K: int, m: int, sms: int = 148) -> int:
    """K slices the listener step gives an [m x O x K] GEMM (csrc/gemm_tc.cu
    gemm_pick_splits and the step's rule in make_op: split only while the tiles
    fill fewer than half of the SMs)."""
    tiles = (O // 128) * -(-m // token_tile(O, m, sms))
    if tiles * 2 >= sms:
        return 1
    total_kb = K // 64
    min_kb = 2 if m <= 128 else 6
    best, best_eff = 1, tiles / (-(-tiles // sms) * sms)
    for s in range(2, 17):
        if total_kb // s < min_kb:
            break
        units = tiles * s
        eff = units / (-(-units // sms) * sms)
        if eff > best_eff + 0.08:
            best, best_eff = s, eff
    return best


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sessions", type=int, default=1024, help="concurrent sessions per GPU")
    ap.add_argument("--weights", default="int8", choices=["int8", "bf16"])
    ap.add_argument("--no-sweep", action="store_true", help="skip the real-time capacity sweep")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-small", action="store_true", help="skip the small-N weight-streaming sweep")
    ap.add_argument("--gemm-probe", type=int, default=0, metavar="M",
                    help="only time the FFN1 GEMM (1536 -> 6144) at M tokens with the weight kind the step "
                         "uses there, and report its HBM GB/s (a small case for kernel profiles)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--cpu-sessions", type=int, default=256,
                    help="sessions of the CPU port's bounded sample of the workload")
    ap.add_argument("--e2e-steps", type=int, default=500, help="end-to-end latency loop length")
    ap.add_argument("--c4-steps", type=int, default=2000, help="config-4 steps (0: skip)")
    ap.add_argument("--c4-sessions", type=int, default=8192, help="config-4 sessions over the whole job")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of this GPU's clocks and throttle reasons during a region."""

    FIELDS = ("pci.bus,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: int | None):
        self.bus_id = bus_id  # PCI bus number of this process's GPU (torch device properties)
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def _mine(self):
        buses = {r[0].lower() for r in self.rows}
        if len(buses) <= 1:
            return self.rows
        def bus(r):
            try:
                return int(r[0], 16)
            except ValueError:
                return -1
        return [r for r in self.rows if self.bus_id is not None and bus(r) == int(self.bus_id)]

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = self._mine()
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------ CPU baseline
def workload_config(args, world: int) -> dict:
    """The workload both arms report (the reference arm times a bounded sample
    of it, described in its cpu_baseline.sample)."""
    n = args.sessions
    return {"workload": f"BASELINE config 3: {n} concurrent ragged sessions/GPU, d=1536 x 12 layers, "
                        f"{args.weights} weights, PCM->mel->Conformer->soft->FiLM",
            "sessions_per_gpu": n, "weights": args.weights,
            "l2": "inputs larger than L2 (0.66 GB weights + KV cache streamed per step)",
            "parallelism": f"session-sharded x{world}"}


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


class CpuPort:
    """The CPU port of the reference path (oracle/: mel + Conformer + FiLM,
    fp32 torch on every host core), driven like the serving tick."""

    def __init__(self, eff: dict):
        import torch
        sys.path.insert(0, str(ROOT))
        from oracle import conformer_ref
        from gemma4_omni_b200.config import FULL

        torch.set_num_threads(host_cores())
        self.cfg = conformer_ref.OracleConfig(hidden=FULL.hidden, layers=FULL.layers, heads=FULL.heads,
                                              ffn=FULL.ffn)
        self.model = conformer_ref.OracleConformer(
            {k: torch.from_numpy(np.asarray(v)) for k, v in eff.items() if not k.startswith("film.")}, self.cfg)
        self.film = {k[5:]: torch.from_numpy(np.asarray(v)) for k, v in eff.items() if k.startswith("film.")}

    def time_steps(self, n: int, steps: int, seconds: float) -> tuple[float, int]:
        """ms per step of n sessions (one untimed warm-up step, then up to
        `steps` timed steps or `seconds`, at least one)."""
        import torch
        from oracle import conformer_ref, film_ref, mel_ref
        from gemma4_omni_b200 import synthetic
        from gemma4_omni_b200.config import FULL

        P = 4
        pcm = np.stack([synthetic.session_audio(99, s, P, total_frames=P) for s in range(n)], axis=1)
        q = torch.randn(n, 2, FULL.film_query_dim)
        state = conformer_ref.zero_state(self.cfg, n)
        tails = [None] * n
        mask = torch.ones(n, 8, dtype=torch.bool)
        done, t0 = -1, 0.0
        while True:
            if done == 0:
                t0 = time.perf_counter()
            mels = []
            for i in range(n):
                m, tails[i] = mel_ref.extract_single_frame(pcm[(done + 1) % P, i], tails[i])
                mels.append(m)
            _, soft, _, _, state = self.model.step(torch.from_numpy(np.stack(mels)), mask, state,
                                                   torch.full((n,), done < 0))
            film_ref.film_forward(self.film, soft, q)
            done += 1
            if done >= 1 and (done >= steps or time.perf_counter() - t0 >= seconds):
                break
        return (time.perf_counter() - t0) / done * 1e3, done


def cpu_baseline(eff: dict, sessions: int, steps: int, seconds: float, ladder: bool) -> dict:
    """The CPU port on the benched workload (`sessions` concurrent sessions,
    a bounded number of steps) and, with `ladder`, ms/step at N in {1,2,4,8,16}
    and the CPU real-time ceiling (largest N with a step under 80 ms)."""
    port = CpuPort(eff)
    ms, done = port.time_steps(sessions, steps, seconds)
    out = {"value": sessions / (ms / 1e3), "unit": UNIT, "cores": host_cores(), "kind": "port",
           "sample": f"{done} timed steps (+1 warm-up) of {sessions} concurrent sessions (a bounded sample of "
                     f"the workload's sessions), d=1536 int8-dequantised tower + mel + FiLM in fp32 "
                     f"({ms:.1f} ms/step)",
           "ms_per_step": ms}
    if ladder:
        per_n = {}
        for n in (1, 2, 4, 8, 16):
            per_n[n] = port.time_steps(n, 20, 2.0)[0]
        ok = [n for n, v in per_n.items() if v < 80.0]
        out["ms_per_step_by_n"] = {str(k): round(v, 2) for k, v in per_n.items()}
        out["realtime_sessions"] = max(ok) if ok else 0
    return out


def synth_weights(pkg, seed=1234):
    from gemma4_omni_b200 import synthetic
    from gemma4_omni_b200.config import FULL
    return synthetic.synthetic_tower_weights(FULL, seed), synthetic.synthetic_film_weights(FULL, seed + 1)


def effective_only(pkg, fmt: int, tower, film):
    from gemma4_omni_b200 import weights
    from gemma4_omni_b200.config import FULL
    return weights.prepare(FULL, tower, film, fmt)[1]


# --------------------------------------------------------------- workload
class Schedule:
    """Per-step rows of `sessions` lanes (BASELINE configs 3-4 arrivals): lane l
    runs sessions back to back, so it is the session's directory handle; the
    handles of lanes whose session ended are released before the next pack.
    Global session ids are lane-local ids * id_stride + id_offset, i.e. the ids
    sharding.shard_of routes to this rank when offset = rank, stride = world."""

    def __init__(self, pkg, sessions: int, steps: int, seed: int, id_offset: int = 0, id_stride: int = 1):
        from gemma4_omni_b200 import synthetic
        ar = synthetic.ArrivalProcess(sessions, seed=seed, mode="lanes")
        self.n = sessions
        self.frames = np.empty((steps, sessions), np.int64)
        self.released: list[np.ndarray] = []
        self.gids: list[np.ndarray] = []
        for t in range(steps):
            lanes, sids, frames, new = ar.step()
            self.frames[t] = frames
            self.released.append(lanes[new].astype(np.int32))
            self.gids.append(sids * id_stride + id_offset)
        self.handles = np.arange(sessions, dtype=np.int32)
        self.keys = np.zeros(sessions, np.int64)

    def device(self, device):
        import torch
        self.d_handles = torch.from_numpy(self.handles).to(device)
        self.d_keys = torch.from_numpy(self.keys).to(device)
        self.d_frames = torch.from_numpy(self.frames).to(device)
        self.d_released = [torch.from_numpy(r).to(device) for r in self.released]
        return self


def pcm_pool(n: int, P: int, device=None):
    from gemma4_omni_b200 import synthetic
    pool = np.stack([synthetic.session_audio(3, s % 4096, P, total_frames=P) for s in range(n)], axis=1)
    return pool if device is None else __import__("torch").from_numpy(pool).to(device)


def device_loop(eng, sched, pcm, query, steps: int, first: int, stream, clocks=None):
    """`steps` device-resident ticks (release -> pack -> step -> commit) from step
    `first`; returns (elapsed ms, sorted per-step ms) from CUDA events."""
    import torch
    P = pcm.shape[0]
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    b.record(stream)
    for i in range(steps):
        t = first + i
        starts[i].record(stream)
        eng.reset_handles(sched.d_released[t])
        f = sched.d_frames[t]
        eng.pack(sched.d_handles, sched.d_keys, f, f)
        eng.step(pcm[t % P], query=query[t % query.shape[0]] if query is not None else None, want_raw=False)
        eng.commit()
        ends[i].record(stream)
    e.record(stream)
    torch.cuda.synchronize()
    return b.elapsed_time(e), sorted(s.elapsed_time(x) for s, x in zip(starts, ends))


def pct(v, q):
    return v[min(len(v) - 1, int(q * len(v)))]


def run_ours(args, pkg, rank, world, device):
    import torch
    from gemma4_omni_b200 import runtime, synthetic
    from gemma4_omni_b200.config import FULL

    fmt = 1 if args.weights == "int8" else 0
    n = args.sessions
    one_gpu = world == 1
    sweep = [] if (args.no_sweep or not one_gpu) else [256, 1024, 2048, 4096, 8192]
    c4_n = args.c4_sessions // world if args.c4_steps > 0 else 0
    cap = max([n, c4_n, 16] + sweep)
    eng = runtime.ListenerEngine(FULL, max_sessions=cap, max_rows=cap, max_handles=cap, weight_format=fmt,
                                 device=device)
    tower, film = synth_weights(pkg)
    eng.load_weights(tower, film, keep_effective=(rank == 0 and one_gpu and not args.no_cpu))
    stream = torch.cuda.current_stream(device)
    P = 4
    total = args.warmup + args.steps
    sched = Schedule(pkg, n, total, seed=7 + rank, id_offset=rank, id_stride=world).device(device)
    pool = pcm_pool(n, P)
    dev_pcm = torch.from_numpy(pool).to(device)
    q_pool = (torch.randn(2, n, 2, FULL.film_query_dim, generator=torch.Generator().manual_seed(rank))
              .to(torch.bfloat16))
    dev_q = q_pool.to(device)

    # ---- warm-up, then the timed region (device-resident inputs)
    device_loop(eng, sched, dev_pcm, dev_q, args.warmup, 0, stream)
    if eng.status() != 0:
        raise RuntimeError(f"device status {eng.status()} after warm-up")
    kernels_per_step = eng.lib.lb_step_kernel_count(eng._ctx) + 3  # graph + release + pack + commit
    bus = None
    try:
        bus = torch.cuda.get_device_properties(device).pci_bus_id
    except Exception:
        pass
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(bus) as clk:
        elapsed_ms, lat = device_loop(eng, sched, dev_pcm, dev_q, args.steps, args.warmup, stream)
    if world > 1:
        torch.distributed.barrier()
    frames = n * args.steps
    if eng.status() != 0:
        raise RuntimeError(f"device status {eng.status()} in the timed region")
    eng.reset_handles(sched.d_handles)

    # ---- end to end through the C ABI with host buffers (lb_step_host), in
    # page-locked memory as a serving process holds its per-tick staging
    def pinned_np(shape, dtype):
        t = torch.empty(shape, dtype={np.uint16: torch.int16, np.float32: torch.float32}[dtype], pin_memory=True)
        return t.numpy().view(dtype)

    def e2e_run(ns, steps, seed, pcm_np, qs):
        sc = Schedule(pkg, ns, steps + 2, seed=seed, id_offset=rank, id_stride=world)
        soft_out = pinned_np((ns, 2, FULL.text_hidden), np.uint16)
        film_out = pinned_np((ns, 2, FULL.film_query_dim), np.uint16)
        pcm_h = []
        for i in range(pcm_np.shape[0]):
            buf = pinned_np((ns, 1280), np.float32)
            buf[...] = pcm_np[i][:ns]
            pcm_h.append(buf)
        q_h = []
        for q in qs:
            buf = pinned_np((ns, 2, FULL.film_query_dim), np.uint16)
            buf[...] = q[:ns].view(torch.int16).numpy().view(np.uint16)
            q_h.append(buf)
        rel_dev = [torch.from_numpy(r).to(device) for r in sc.released]
        lats = []
        t_all = 0.0
        for t in range(steps + 2):
            a = time.perf_counter()
            eng.reset_handles(rel_dev[t])
            eng.step_host(sc.handles, sc.keys, sc.frames[t], sc.frames[t], pcm_h[t % len(pcm_h)],
                          query=q_h[t % len(q_h)], out_soft=soft_out, out_film=film_out)
            dt = time.perf_counter() - a
            if t >= 2:
                lats.append(dt * 1e3)
                t_all += dt
        torch.cuda.synchronize(device)
        eng.reset_handles(torch.from_numpy(sc.handles).to(device))
        h2d = int(sc.handles.nbytes + sc.keys.nbytes + 2 * sc.frames[0].nbytes + pcm_h[0].nbytes + q_h[0].nbytes)
        d2h = int(soft_out.nbytes + film_out.nbytes)
        return sorted(lats), ns * steps / t_all, h2d, d2h

    if world > 1:
        torch.distributed.barrier()
    e2e_lat, e2e_value, h2d, d2h = e2e_run(n, args.e2e_steps, 1000 + rank, pool, list(q_pool))

    # ---- dominant kernel: the FFN1 GEMM at this step's token count, timed alone,
    # with the weight kind and K split the step's bucket uses: int8 codes read as
    # fp16-widened codes from wide_min_tokens() tokens on (w_kind 2), in-kernel
    # widening below (w_kind 1)
    M = 2 * n
    w_kind = fmt
    if fmt == 1 and M >= wide_min_tokens() and os.environ.get("LB_INT8_WIDE", "1") != "0":
        w_kind = 2
    splits = step_splits(FULL.ffn, FULL.hidden, M)
    x = torch.randn(M, FULL.hidden, device=device).to(torch.float16 if fmt == 1 else torch.bfloat16)
    if fmt == 1:
        wq = torch.randint(-127, 128, (FULL.ffn, FULL.hidden), dtype=torch.int8, device=device)
        if w_kind == 2:
            wq = wq.to(torch.float16)
        sc_ = torch.full((FULL.ffn,), 1e-3, dtype=torch.float16, device=device)
    else:
        wq = (torch.randn(FULL.ffn, FULL.hidden, device=device) * 0.02).to(torch.bfloat16)
        sc_ = None
    yo = torch.empty(M, FULL.ffn, dtype=torch.bfloat16, device=device)
    # a split GEMM reduces through this zeroed workspace and a finish pass
    acc_ = torch.zeros(M, FULL.ffn, device=device) if splits > 1 else None

    def gemm():
        rc = eng.lib.lb_op_gemm_clipped(x.data_ptr(), FULL.hidden, M, 0, wq.data_ptr(), w_kind,
                                        None if sc_ is None else sc_.data_ptr(), None, FULL.ffn, FULL.hidden,
                                        yo.data_ptr(), FULL.ffn, 0, 1, splits, 1, None, None,
                                        None if acc_ is None else acc_.data_ptr(), None, stream.cuda_stream)
        assert rc == 0, rc
    for _ in range(5):
        gemm()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    reps = 50
    for _ in range(reps):
        gemm()
    g1.record(stream)
    torch.cuda.synchronize(device)
    gemm_ms = g0.elapsed_time(g1) / reps
    del x, wq, yo, acc_

    # ---- weight-streaming regime: small N, device-resident, step time vs the
    # step's algorithmic bytes (weights + per-session state)
    small = {}
    if one_gpu and not args.no_small:
        for ns in (1, 4, 16, 64):
            sc = Schedule(pkg, ns, 230, seed=300 + ns).device(device)
            pc = dev_pcm[:, :ns].contiguous()
            qq = dev_q[:, :ns].contiguous()
            device_loop(eng, sc, pc, qq, 30, 0, stream)
            ms_all, lats = device_loop(eng, sc, pc, qq, 200, 30, stream)
            eng.reset_handles(sc.d_handles)
            ms = ms_all / 200
            nbytes = (0.659e9 if fmt == 1 else 1.318e9) + ns * 1.24e6
            small[str(ns)] = {"ms_per_step": ms, "p50_ms": pct(lats, 0.5), "p99_ms": pct(lats, 0.99),
                              "frames_per_s": ns / (ms / 1e3), "algorithmic_bytes": nbytes,
                              "achieved_gbs": nbytes / (ms / 1e3) / 1e9}

    # ---- real-time capacity sweep (1 GPU), end to end: largest N with p99 < 20 ms
    sweep_res = {}
    if sweep:
        big_pool = pcm_pool(max(sweep), 2)
        big_q = [torch.randn(max(sweep), 2, FULL.film_query_dim).to(torch.bfloat16) for _ in range(2)]
        for ns in sweep:
            lats, fps, _, _ = e2e_run(ns, 100, 50 + ns, big_pool, big_q)
            sweep_res[str(ns)] = {"p50_ms": pct(lats, 0.5), "p99_ms": pct(lats, 0.99), "frames_per_s": fps,
                                  "steps": 100, "path": "lb_step_host (copies included)"}
        del big_pool, big_q
        if eng.status() != 0:
            raise RuntimeError("device status error in the sweep")

    # ---- c4_sessions in total, sharded by session id over
    # the job's ranks (strong scaling), args.c4_steps device-resident steps
    c4 = None
    if c4_n:
        sc = Schedule(pkg, c4_n, args.c4_steps + 5, seed=4000 + rank, id_offset=rank, id_stride=world).device(device)
        pc = torch.from_numpy(pcm_pool(c4_n, 2)).to(device)
        qq = torch.randn(2, c4_n, 2, FULL.film_query_dim, device=device).to(torch.bfloat16)
        device_loop(eng, sc, pc, qq, 5, 0, stream)
        if world > 1:
            torch.distributed.barrier()
        c4_ms, c4_lat = device_loop(eng, sc, pc, qq, args.c4_steps, 5, stream)
        eng.reset_handles(sc.d_handles)
        c4 = {"elapsed_ms": c4_ms, "frames": c4_n * args.c4_steps, "p50": pct(c4_lat, 0.5),
              "p99": pct(c4_lat, 0.99), "sessions_per_gpu": c4_n}
        del sc, pc, qq
        if eng.status() != 0:
            raise RuntimeError("device status error in config 4")

    eff = eng.effective_weights
    eng.close()
    return dict(elapsed_ms=elapsed_ms, lat=lat, frames=frames, kernels=kernels_per_step,
                clocks=clk.summary(), e2e_value=e2e_value, e2e_lat=e2e_lat, h2d=h2d, d2h=d2h, gemm_ms=gemm_ms, M=M,
                w_kind=w_kind, gemm_splits=splits, sweep=sweep_res, small=small, c4=c4, eff=eff)


def step_roofline_ms(n: int, weights: str, peaks: dict) -> float:
    """BASELINE step roofline: max(N x 2.644 GFLOP / sustained tensor peak,
    (W + N x 1.24 MB) / HBM peak)."""
    W = 0.659e9 if weights == "int8" else 1.318e9
    return 1e3 * max(n * 2.644e9 / (peaks.get("bf16_tflops_sustained", 1390.3) * 1e12),
                     (W + n * 1.24e6) / (peaks.get("hbm_gbs", 6650.0) * 1e9))


def gemm_probe(args, pkg) -> dict:
    """The step's FFN1 GEMM alone at M tokens (int8: in-kernel widening below
    wide_min_tokens(), fp16 codes from there) with 1 and 3 K slices (3: through
    a workspace and a finish pass), timed with CUDA events on its stream;
    algorithmic bytes = weights (+ scales) + activations in + outputs out."""
    import torch
    from gemma4_omni_b200 import _lib
    from gemma4_omni_b200.config import FULL

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M, O, K = args.gemm_probe, FULL.ffn, FULL.hidden
    int8 = args.weights == "int8"
    w_kind = (2 if M >= wide_min_tokens() else 1) if int8 else 0
    x = torch.randn(M, K, device=dev).to(torch.float16 if int8 else torch.bfloat16)
    if int8:
        w = torch.randint(-127, 128, (O, K), dtype=torch.int8, device=dev)
        if w_kind == 2:
            w = w.to(torch.float16)
        sc = torch.full((O,), 1e-3, dtype=torch.float16, device=dev)
    else:
        w, sc = (torch.randn(O, K, device=dev) * 0.02).to(torch.bfloat16), None
    y = torch.empty(M, O, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    # the step's split count for this shape (SMs filled by K slices)
    acc = torch.zeros(M, O, device=dev)

    def run(splits):
        rc = lib.lb_op_gemm_clipped(x.data_ptr(), K, M, 0, w.data_ptr(), w_kind, None if sc is None else sc.data_ptr(),
                                    None, O, K, y.data_ptr(), O, 0, 1, splits, 1, None, None,
                                    acc.data_ptr() if splits > 1 else None, None, stream.cuda_stream)
        assert rc == 0
    out = {"M": M, "w_kind": w_kind, "per_splits": {}}
    for splits in (1, 3):
        for _ in range(5):
            run(splits)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(50):
            run(splits)
        b.record(stream)
        torch.cuda.synchronize(dev)
        us = a.elapsed_time(b) / 50 * 1e3
        nbytes = w.numel() * w.element_size() + (O * 2 if int8 else 0) + x.numel() * 2 + y.numel() * 2
        out["per_splits"][str(splits)] = {"us": us, "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / us / 1e3}
    return out


def main():
    args = parse()
    pkg = load_package()
    if args.gemm_probe:
        print(json.dumps({"gemm_probe": gemm_probe(args, pkg)}), flush=True)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dtype = "int8w-fp16act" if args.weights == "int8" else "bf16w-fp16act"
    if args.impl == "reference":
        if rank != 0:
            return
        tower, film = synth_weights(pkg)
        eff = effective_only(pkg, 1 if args.weights == "int8" else 0, tower, film)
        del tower, film
        cpu = cpu_baseline(eff, min(args.cpu_sessions, args.sessions), 3, max(args.cpu_seconds, 10.0),
                           ladder=False)
        line = {"impl": "reference", "metric": METRIC, "value": cpu["value"], "unit": UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": cpu["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": workload_config(args, args.gpus),
                "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cpu["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=device)
    res = run_ours(args, pkg, rank, world, device)
    elapsed_ms, frames = res["elapsed_ms"], res["frames"]
    e2e_value = res["e2e_value"]
    lat = res["lat"]
    p50, p99 = pct(lat, 0.5), pct(lat, 0.99)
    e2e_p50, e2e_p99 = pct(res["e2e_lat"], 0.5), pct(res["e2e_lat"], 0.99)
    c4 = res["c4"]
    c4_vals = [c4["elapsed_ms"], c4["p50"], c4["p99"]] if c4 else [0.0, 0.0, 0.0]
    c4_frames = c4["frames"] if c4 else 0
    e2e_time = args.sessions * args.e2e_steps / e2e_value
    if world > 1:
        from gemma4_omni_b200 import sharding
        # whole job: the slowest rank's times, every rank's frames
        times, counts = sharding.reduce_over_ranks(
            [elapsed_ms, e2e_time, p50, p99, e2e_p50, e2e_p99] + c4_vals,
            [frames, args.sessions * args.e2e_steps, c4_frames], device=device)
        elapsed_ms, e2e_time, p50, p99, e2e_p50, e2e_p99 = times[:6]
        c4_vals = times[6:]
        frames, e2e_frames, c4_frames = counts
        e2e_value = e2e_frames / e2e_time
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu and res["eff"] is not None:
        # after the GPU work and outside any process group: all host cores, N=1 job only
        cpu = cpu_baseline(res["eff"], min(args.cpu_sessions, args.sessions), 2, args.cpu_seconds, ladder=True)
    from gemma4_omni_b200.config import FULL
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak_tf = peaks.get("bf16_tflops", 1590.0)
    peak_src = "measured" if peaks else "fallback"
    hbm = peaks.get("hbm_gbs", 6650.0)
    value = frames / (elapsed_ms / 1e3)
    ms_step = elapsed_ms / args.steps
    M = res["M"]
    gemm_flops = 2.0 * M * FULL.ffn * FULL.hidden
    # algorithmic bytes of the launch: weights (int8 codes, or their fp16
    # widening) + fp16 scales + fp16 activations in + bf16 outputs
    w_bytes = FULL.ffn * FULL.hidden * (2 if res["w_kind"] != 1 else 1)
    gemm_bytes = w_bytes + 2 * FULL.ffn + 2 * M * FULL.hidden + 2 * M * FULL.ffn
    # the roof that binds this shape: tensor throughput or the weight stream
    tensor_bound = gemm_flops / (peak_tf * 1e12) >= gemm_bytes / (hbm * 1e9)
    if tensor_bound:
        achieved = gemm_flops / (res["gemm_ms"] * 1e-3) / 1e12
    else:
        achieved = gemm_bytes / (res["gemm_ms"] * 1e-3) / 1e9
    # DRAM bytes (read + write) of one launch of this GEMM from an ncu --set full
    # capture of the same shape and weight kind (M=2048, fp16 activations): W and
    # X are read once; the 25 MB output stays in L2 by kernel end.
    traffic, traffic_src = None, None
    if M == 2048 and args.weights == "int8":
        # in-kernel widening reads 9.4 MB of int8 codes, fp16 codes 18.9 MB (+ 6.3 MB X)
        traffic = {1: 15.794432e6, 2: 25.478144e6}.get(res["w_kind"])
        traffic_src = "ncu dram__bytes_read.sum + dram__bytes_write.sum, bytes per launch"
    t_roof = step_roofline_ms(args.sessions, args.weights, peaks)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded PCM, N(0,0.02) weights, geometric session arrivals)",
        "config": workload_config(args, world),
        "latency_ms": {"p50": p50, "p99": p99, "max": lat[-1], "steps": len(lat), "path": "device-resident"},
        "roofline": {"bound": "tensor" if tensor_bound else "hbm",
                     "kernel": f"FFN1 GEMM {M}x{FULL.ffn}x{FULL.hidden}, weights "
                     + {0: "bf16", 1: "int8 (widened in-kernel)", 2: "int8 codes widened to fp16"}[res["w_kind"]]
                     + (f", {res['gemm_splits']} K slices" if res["gemm_splits"] > 1 else ""),
                     "achieved": achieved, "peak": peak_tf if tensor_bound else hbm,
                     "unit": "TFLOP/s" if tensor_bound else "GB/s",
                     "frac": achieved / (peak_tf if tensor_bound else hbm),
                     "algorithmic": gemm_flops if tensor_bound else gemm_bytes,
                     "traffic": traffic, "traffic_source": traffic_src,
                     "peak_source": (f"{peak_src} bf16 burst (kernel timed alone)" if tensor_bound
                                     else f"{peak_src} HBM copy bandwidth")},
        "roofline_step": {"t_roof_ms": t_roof, "t_measured_ms": ms_step, "frac": t_roof / ms_step,
                          "definition": "max(N*2.644 GFLOP / sustained bf16 peak, (W + N*1.24 MB) / HBM peak)"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"],
                "steps": args.e2e_steps},
        "latency_e2e_ms": {"p50": e2e_p50, "p99": e2e_p99, "steps": args.e2e_steps,
                           "path": "lb_step_host, host buffers, copies and release/pack/commit included"},
        "clocks": res["clocks"],
        "gpu_launches": int(res["kernels"] * args.steps),
        "gpu_launches_per_step": res["kernels"],
    }
    if res["small"]:
        for v in res["small"].values():
            v["hbm_frac"] = v["achieved_gbs"] / hbm
        line["small_n"] = {"regime": "weight streaming (HBM-bound below ~80 sessions at int8)",
                           "hbm_peak_gbs": hbm, "per_n": res["small"],
                           "bytes_definition": "W + N x 1.24 MB per step (weights + per-session state)"}
    if res["sweep"]:
        ok = [int(ns) for ns, v in res["sweep"].items() if v["p99_ms"] < 20.0]
        line["realtime_sessions_per_gpu"] = max(ok) if ok else 0
        line["capacity_sweep"] = res["sweep"]
    if c4:
        c4_ms, c4_p50, c4_p99 = c4_vals
        per_gpu = args.c4_sessions // world
        c4_step = c4_ms / args.c4_steps
        line["config4"] = {"sessions_total": args.c4_sessions, "sessions_per_gpu": per_gpu, "steps": args.c4_steps,
                           "frames_per_s": c4_frames / (c4_ms / 1e3), "ms_per_step": c4_step,
                           "p50_ms": c4_p50, "p99_ms": c4_p99,
                           "roofline_frac_per_gpu": step_roofline_ms(per_gpu, args.weights, peaks) / c4_step,
                           "realtime": c4_p99 < 20.0, "scaling": "strong (fixed total sessions)",
                           "path": "device-resident, max over ranks"}
    if cpu:
        line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line["cpu_baseline"]["ms_per_step_by_n"] = cpu["ms_per_step_by_n"]
        line["cpu_baseline"]["realtime_sessions"] = cpu["realtime_sessions"]
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
