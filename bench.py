"""Benchmark of the action-expert Euler loop, steps 2-10 (BASELINE.json metric):
"action-expert ms per predict (steps 2-10, batch 1, 1xB200); episodes/s at 1/2/4/8 GPUs".

    python bench.py [--gpus N --steps K --warmup W] [--impl mk|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

One step = one predict's Euler steps 2..10 for one episode (REKI's expert,
bf16, batch 1, T = 10 action rows, 2 of 3 register frames valid, 160 cross-attention source rows),
replayed as a CUDA graph like the reference's own timing (src/profile_breakdown.py:107-130).
Multi-GPU: one process per GPU, each serving its own episodes with its own weights copy, no
collective (the path does not shard); value = episodes/s summed over ranks, from the max over
ranks of the per-step device time.

``--impl reference`` times the reference algorithm's CPU implementation on this host's cores: the
repo's CPU oracle in fp32 (Kyutai's eager expert is not available here; the oracle restates it),
rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "action-expert ms per predict (steps 2–10, batch 1, 1×B200); episodes/s at 1/2/4/8 GPUs"
PUBLISHED_MS = 4.00          # reference megakernel v5, steps 2-10, 1x B200 (results/gpus/b200/test_mk.json:16)
HBM_FALLBACK_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20


def algorithmic_bytes_per_step(dims, mods_row_bytes: int) -> int:
    """HBM bytes one Euler step must stream: bf16 weights + fp32 in/out projections + norm weights +
    one modulation row, 212,678,400 B at the BASELINE configs[1] shapes (bf16 modulation row)."""
    L, H, I, A, HD = dims.L, dims.H, dims.I, dims.A, dims.HD
    bf16 = 2 * L * (3 * H * H + 3 * H * H + 3 * H * I)
    fp32 = 4 * (2 * A * H)
    norms = 2 * 3 * L * HD
    return bf16 + fp32 + norms + mods_row_bytes


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return HBM_FALLBACK_GBS, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"mkx_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = [r.split(",") for r in self.path.read_text().splitlines() if r.strip()]
        self.path.unlink(missing_ok=True)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


KERNEL_SOURCES = ("reki_megakernel_b200/csrc/mk_expert.cu", "reki_megakernel_b200/csrc/mkx_device.cuh")


def kernel_source_sha() -> str:
    """sha256 (first 16 hex digits) of the expert kernel's sources, as recorded in the ncu summary."""
    import hashlib
    h = hashlib.sha256()
    for f in KERNEL_SOURCES:
        h.update((ROOT / f).read_bytes())
    return h.hexdigest()[:16]


def traffic_from_profile():
    """(dram bytes read + written per launch of expert_kernel, source note) from the committed ncu
    summary, or (None, why) when the summary was captured from other kernel sources than these."""
    p = ROOT / "profiles" / "expert_kernel_full.md"
    if not p.exists():
        return None, "no ncu summary"
    traffic, sha = None, None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                traffic = int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                traffic = None
        if line.startswith("kernel_source_sha16:"):
            sha = line.split(":", 1)[1].strip().split()[0]
    if sha != kernel_source_sha():
        return None, f"ncu summary captured from other kernel sources ({sha}), not these ({kernel_source_sha()})"
    return traffic, f"ncu capture of these kernel sources (sha {sha}), profiles/expert_kernel_full.md"


# ------------------------------------------------------------------------------------------------
def cpu_predict_ms(dims, S: int, threads: int, warmup: int, min_n: int, seconds: float):
    """fp32 eager CPU expert (the oracle), whole predicts (Euler steps 2..10 of one episode) on this
    host's cores; returns the per-predict times in ms (at least min_n, or until `seconds` elapsed)."""
    from oracle.expert_oracle import OracleExpert
    from reki_megakernel_b200.synthetic import make_inputs, make_weights
    torch.set_num_threads(threads)
    orc = OracleExpert(make_weights(dims, seed=0), "fp32")
    inp = make_inputs(dims, n_steps=9, S=S)
    e = inp.episode(0)
    ep = dict(x=e.x[0], mods=e.mods[0], dt=e.dt[0], memk=e.memk[0], memv=e.memv[0], kv_start=int(e.kv_start[0]),
              kca=e.kca[0], vca=e.vca[0], S=int(e.S[0]), sa_cos=e.sa_cos[0], sa_sin=e.sa_sin[0],
              ca_cos=e.ca_cos[0], ca_sin=e.ca_sin[0], action_dim=inp.action_dim)
    for _ in range(warmup):
        orc.run_episode(ep)
    times, t0 = [], time.perf_counter()
    while len(times) < min_n or (seconds > 0 and time.perf_counter() - t0 < seconds):
        a = time.perf_counter()
        orc.run_episode(ep)
        times.append((time.perf_counter() - a) * 1e3)
    return times


def bench_config(args, world: int) -> dict:
    """The workload description shared by both arms (the reference arm runs the same workload on the
    host cores)."""
    return {"workload": "REKI expert Euler steps 2-10 (BASELINE configs[1]); one step = one predict of each "
                        "of this GPU's episodes, batch-1 launches back to back",
            "T": 10, "S": args.S, "memory_rows": 64, "euler_steps": 9, "episodes_per_gpu": args.batch,
            "parallelism": f"replicas x{world}, no collective",
            "l2": "256 MB written between timed steps (untimed); weights (212 MB/Euler step) exceed L2",
            "timing": "CUDA-graph replay, CUDA events per step, mean over steps, max over ranks"}


def run_reference(args, rank: int, world: int):
    """The reference algorithm's CPU implementation (the fp32 oracle: Kyutai's eager expert is not
    available here) on all host cores, rank 0 only: `--warmup` untimed then `--steps` timed whole
    predicts (capped at --max-ref-steps), median per predict."""
    if rank != 0:
        return
    from reki_megakernel_b200.synthetic import ExpertDims
    dims = ExpertDims()
    threads = len(os.sched_getaffinity(0))
    steps = min(args.steps, args.max_ref_steps)
    times = cpu_predict_ms(dims, args.S, threads, args.warmup, steps, 0.0)
    ms_predict = statistics.median(times)
    value = 1000.0 / ms_predict
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "episodes/s", "n_gpus": args.gpus,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": ms_predict, "ms_per_predict": ms_predict,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded weights, BASELINE configs[1] shapes)",
        "config": bench_config(args, world),
        "cpu_baseline": {"value": value, "unit": "episodes/s", "cores": threads, "kind": "port",
                         "sample": f"{len(times)} whole predicts (9 Euler steps each) of one episode, fp32 CPU oracle, "
                                   "median"},
        "e2e": {"value": value, "unit": "episodes/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s_timed_region": sum(times) / 1e3,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
STAGE_NAMES = ["qkv", "sa", "o", "ca_q", "ca", "ca_o", "gate_up", "down"]


def run_timeline(args):
    """Per-stage critical path of one predict from the kernel's stage stamps
    (thread 0 of every CTA stamps %globaltimer at the end of each stage, as the reference's PROFILE
    mode does): for each stage, end of the last CTA minus end of the last CTA in the previous stage,
    median over layers and Euler steps. Not a bench line: the stamps add a store per stage."""
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_past, make_weights
    dims = ExpertDims()
    mk = ExpertMegakernel(weights=make_weights(dims, seed=0).to("cuda"))
    inp = make_inputs(dims).to("cuda")
    past = make_past(inp)
    n = inp.n_steps
    stride = 1 + mk.barriers(n)
    prof = torch.zeros(mk.nprog * stride, dtype=torch.int64, device="cuda")
    runs = []
    for _ in range(args.warmup + args.steps):
        prof.zero_()
        mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], past, inp.action_dim, prof=prof)
        torch.cuda.synchronize()
        mk.check_device_error()
        runs.append(prof.view(mk.nprog, stride).cpu())
    per = {}
    for a in runs[args.warmup:]:
        ends = a[:, 1:]
        last = ends.max(dim=0).values
        prev = a[:, 0].min()
        for k in range(ends.shape[1]):
            if k == 0:
                name = "first_tail"
            else:
                j = (k - 1) % (8 * dims.L + 1)
                name = "step_tail" if j == 8 * dims.L else STAGE_NAMES[j % 8]
            per.setdefault(name, []).append(float(last[k] - prev) / 1e3)
            prev = last[k]
    total = [float(a[:, 1:].max() - a[:, 0].min()) / 1e3 for a in runs[args.warmup:]]
    out = {"timeline_us": {k: round(statistics.median(v), 3) for k, v in per.items()},
           "per_layer_us": round(sum(statistics.median(per[k]) for k in STAGE_NAMES), 3),
           "predict_us": round(statistics.median(total), 1), "predicts": len(total),
           "config": "REKI expert steps 2-10, T=10, S=160, 64 memory rows, batch 1"}
    print(json.dumps(out), flush=True)


SUBSTAGE_POINTS = {
    # numbered %globaltimer points inside each stage (thread 0 of the CTA), in the order they fire
    "adarms_gemm": {6: "polls (thread 0's word pairs)", 4: "row sum of squares (the warp has its rows)",
                    1: "AdaRMS arithmetic", 0: "X written", 2: "weight slot wait + barrier",
                    3: "MMA + barrier", 5: "epilogue (publish)", 7: "stage end"},
    "attention": {1: "polls (query, own k/v)", 3: "norm/RoPE + scores + block max",
                  2: "softmax + P.V", 4: "group shuffles + partials to shared", 5: "barrier",
                  7: "final reduce + publish y"},
    "words_gemm": {0: "weight slot wait", 1: "polls + MMA + barrier", 5: "gated-residual epilogue (publish)",
                   6: "barrier", 7: "stage end"},
    "down": {0: "weight slot wait", 1: "level 1: polls of g + MMA + barrier", 2: "level 1 partials published",
             3: "level 2: polls of the group partials + barrier", 5: "sum + gated residual (publish h)",
             6: "barrier", 7: "stage end"},
}
SUBSTAGE_FAMILY = {"qkv": "adarms_gemm", "ca_q": "adarms_gemm", "gate_up": "adarms_gemm", "sa": "attention",
                   "ca": "attention", "o": "words_gemm", "ca_o": "words_gemm", "down": "down"}


def run_substage(args):
    """Sub-phases of every layer stage, from the profiling build of the kernel (``libmkx_trace.so``,
    compiled with -DMKX_SUBSTAGE_TRACE): thread 0 of CTA 0 stamps %globaltimer at numbered points
    inside each stage. Per stage and point, in the order the points fire: time since the previous
    point, the first measured from the end of the last CTA in the previous stage; median over the
    90 layer passes and the predicts. Not a bench line: the stamps add stores."""
    from reki_megakernel_b200 import _lib
    _lib.use_traced_build()
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_past, make_weights
    dims = ExpertDims()
    mk = ExpertMegakernel(weights=make_weights(dims, seed=0).to("cuda"))
    inp = make_inputs(dims).to("cuda")
    past = make_past(inp)
    G, n = mk.nprog, inp.n_steps
    per = 1 + mk.barriers(n)
    prof = torch.zeros(G * per + 16 * per, dtype=torch.int64, device="cuda")  # stage ends + 2 CTAs x 8 points
    acc, stage_us = {}, {}
    for it in range(args.warmup + args.steps):
        prof.zero_()
        mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], past, inp.action_dim, prof=prof)
        torch.cuda.synchronize()
        mk.check_device_error()
        if it < args.warmup:
            continue
        a = prof.cpu()
        last = a[:G * per].view(G, per).max(0).values  # [1 + stage]: end of the last CTA
        sub = a[G * per: G * per + 8 * per].view(per, 8)  # CTA 0: [stage index][point]
        for s in range(n):
            for l in range(dims.L):
                for k, name in enumerate(STAGE_NAMES):
                    st = 1 + s * (8 * dims.L + 1) + 8 * l + k  # stages finished before this one
                    t0 = int(last[st])
                    for v, pt in sorted((int(sub[st, q]), q) for q in range(8) if int(sub[st, q]) != 0):
                        acc.setdefault((name, pt), []).append((v - t0) / 1e3)
                        t0 = v
                    stage_us.setdefault(name, []).append(float(last[st + 1] - last[st]) / 1e3)
    out = {}
    for name in STAGE_NAMES:
        pts = SUBSTAGE_POINTS[SUBSTAGE_FAMILY[name]]
        order = [q for q in pts if (name, q) in acc]
        out[name] = {"stage_us": round(statistics.median(stage_us[name]), 3),
                     "points": [[pts[q], round(statistics.median(acc[(name, q)]), 3)] for q in order]}
    print(json.dumps({"substage_us": out, "cta": 0, "predicts": args.steps,
                      "config": "REKI expert steps 2-10, T=10, S=160, 64 memory rows, batch 1"}), flush=True)


def run_predict(args):
    """The GPU half of one predict after Euler step 1 (BASELINE configs[2] without step 1 and the VLM):
    modulation rows, cross-attention K/V of all layers and Euler steps 2..N replayed as one CUDA graph
    (PredictGraph). Prints one JSON line (not the headline metric)."""
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.modulations import StepModulations
    from reki_megakernel_b200.predict import PredictGraph
    from reki_megakernel_b200.prepare import RegisterPrepare
    from reki_megakernel_b200.synthetic import (ExpertDims, make_inputs, make_modulation_weights, make_prepare_weights,
                                                make_source, make_state, make_weights)
    dims = ExpertDims()
    S = args.S
    mk = ExpertMegakernel(weights=make_weights(dims, seed=0).to("cuda"))
    rp = RegisterPrepare(make_prepare_weights(dims, seed=0).to("cuda"))
    sm = StepModulations(make_modulation_weights(dims, seed=0).to("cuda"))
    inp = make_inputs(dims, S=S).to("cuda")
    pg = PredictGraph(mk, rp, sm, num_steps=10, S=S, T=10, memk=inp.memk[0], memv=inp.memv[0],
                      kv_start=int(inp.kv_start[0]), action_dim=inp.action_dim)
    src = make_source(S, dims.src_dim, seed=0).to("cuda")
    state = make_state(sm.sdim, seed=0).to("cuda")
    x_t = inp.x[:1].contiguous()
    pg(src, state, x_t)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        pg.graph.replay()
    torch.cuda.synchronize()
    pg.check_device_errors()
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.3)
    per = []
    for _ in range(args.steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        pg.graph.replay()
        b.record()
        b.synchronize()
        per.append(a.elapsed_time(b))
    clk = clocks.stop()
    pg.check_device_errors()
    ms = statistics.mean(per)
    L, H = dims.L, dims.H
    wbytes = (9 * algorithmic_bytes_per_step(dims, dims.MODW * 2) + dims.MODW * H * 2 + dims.MODW * 4
              + L * 2 * H * dims.src_dim * 2)
    hbm, peak_kind = peaks()
    achieved = wbytes / (ms * 1e-3) / 1e9
    line = {
        "metric": "GPU half of a predict after step 1: modulations + register_prepare + Euler steps 2-10, ms",
        "value": ms, "unit": "ms", "higher_is_better": False, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "dtype": "bf16", "data": "synthetic (seeded weights and inputs)",
        "config": {"workload": f"one CUDA graph: 10 modulation rows, K/V of {L} layers from S={S} source rows, "
                               "9 Euler steps of the expert", "S": S, "T": 10, "euler_steps": 9,
                   "l2": "256 MB written between timed replays (untimed)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": f"{peak_kind} (hbm copy, burst)", "algorithmic_bytes": wbytes},
        "gpu_launches": 4 * args.steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_full(args):
    """A whole predict: all 10 Euler steps in one persistent launch, the step
    modulations, register_prepare, the register pass of the current frame and the carry of 3 register
    frames x 32 rows, as one CUDA graph (FullPredict), over consecutive seeded predicts. Prints one
    JSON line (not the headline metric)."""
    from reki_megakernel_b200.batch import BatchedExpert
    from reki_megakernel_b200.full_predict import FullPredict
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.modulations import StepModulations
    from reki_megakernel_b200.prepare import RegisterPrepare
    from reki_megakernel_b200.synthetic import (ExpertDims, make_modulation_weights, make_prepare_weights,
                                                make_register_rows, make_source, make_state, make_weights)
    dims = ExpertDims()
    S, R, N, T = args.S, 32, 10, 10
    w = make_weights(dims, seed=0).to("cuda")
    mk = ExpertMegakernel(weights=w)
    bx = BatchedExpert(w, max_episodes=R // 16)
    rp = RegisterPrepare(make_prepare_weights(dims, seed=0).to("cuda"))
    sm = StepModulations(make_modulation_weights(dims, seed=0).to("cuda"))
    fp = FullPredict(mk, bx, rp, sm, make_register_rows(dims, R).to("cuda"), S=S, num_steps=N, T=T)
    n_in = 20  # 20 consecutive seeded predicts, repeated
    ins = [(make_source(S, dims.src_dim, seed=100 + p).to("cuda"), make_state(sm.sdim, seed=100 + p).to("cuda"),
            torch.randn((1, T, dims.A), generator=torch.Generator().manual_seed(1234 + p)).to("cuda"))
           for p in range(n_in)]
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for i in range(args.warmup):
        fp(*ins[i % n_in])
    torch.cuda.synchronize()
    fp.check_device_errors()
    fp.reset()
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.3)
    per = []
    for i in range(args.steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fp(*ins[i % n_in])
        b.record()
        b.synchronize()
        per.append(a.elapsed_time(b))
    clk = clocks.stop()
    fp.check_device_errors()
    L, H, I = dims.L, dims.H, dims.I
    layer_w = L * (3 * H * H + 3 * H * H + 3 * I * H) * 2
    reg_launches = bx.launches(R // 16, 16, 1) - 2  # the pass: per layer the loop's launches (no tails)
    wbytes = (N * algorithmic_bytes_per_step(dims, dims.MODW * 2) + layer_w + dims.MODW * H * 2 + dims.MODW * 4
              + L * 2 * H * dims.src_dim * 2)
    ms = statistics.mean(per)
    hbm, peak_kind = peaks()
    achieved = wbytes / (ms * 1e-3) / 1e9
    line = {
        "metric": "whole predict: 10 Euler steps + modulations + register_prepare + register pass + frame carry, ms",
        "value": ms, "unit": "ms", "higher_is_better": False, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "dtype": "bf16", "data": "synthetic (seeded weights; 20 seeded predicts repeated)",
        "ms_p50": statistics.median(per), "ms_p99": sorted(per)[min(len(per) - 1, int(0.99 * len(per)))],
        "config": {"workload": f"BASELINE configs[2]: one CUDA graph per predict; S={S} source rows x 2048, "
                               f"{R} register rows per frame, 3 frames carried, T={T} action rows, N={N} steps "
                               "in one persistent launch",
                   "S": S, "T": T, "euler_steps": N, "register_rows": R, "frames": 3,
                   "l2": "256 MB written between timed predicts (untimed)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": f"{peak_kind} (hbm copy, burst)", "algorithmic_bytes": wbytes},
        "gpu_launches": (4 + reg_launches) * args.steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_mods(args):
    """Per-step modulation rows of one predict (BASELINE configs[2]'s modulation part): N = 10 rows of
    MODW = 70,656 from the conditioning network, two launches (conditioning + HBM-bound projection).
    Prints one JSON line (not the headline metric)."""
    from reki_megakernel_b200.modulations import StepModulations
    from reki_megakernel_b200.synthetic import ExpertDims, make_modulation_weights, make_state
    dims = ExpertDims()
    N = 10
    w = make_modulation_weights(dims, seed=0)
    st_h = make_state(w.sdim, seed=0)
    sm = StepModulations(w.to("cuda"))
    st = st_h.to("cuda")
    mods, dt = sm(N, st)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        sm(N, st, out=(mods, dt))
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        sm(N, st, out=(mods, dt))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.3)
    per = []
    for _ in range(args.steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        per.append(a.elapsed_time(b))
    clk = clocks.stop()
    ms = statistics.mean(per)
    MODW, H = dims.MODW, dims.H
    wbytes = MODW * H * 2 + MODW * 4 + H * (w.tdim + w.sdim) * 4
    io_bytes = N * MODW * 2
    hbm, peak_kind = peaks()
    achieved = (wbytes + io_bytes) / (ms * 1e-3) / 1e9
    # CPU: the same network in fp32 on the host cores (bf16 weights widened once, outside the timing)
    thr = len(os.sched_getaffinity(0))
    torch.set_num_threads(thr)
    wm = w.w_m.float()
    t0 = time.perf_counter()
    reps = 0
    while reps < 2 or time.perf_counter() - t0 < 5.0:
        half = w.tdim // 2
        t = 1.0 - torch.arange(N, dtype=torch.float32) / N
        f = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32) / half)
        ang = 1000.0 * t[:, None] * f[None, :]
        e = 8.0 * (torch.cat([ang.cos(), ang.sin()], 1) @ w.w_t.T + st_h[None, :] @ w.w_s.T)
        a = torch.nn.functional.silu(e).to(torch.bfloat16).float()
        (a @ wm.T + w.b_m).to(torch.bfloat16)
        reps += 1
    cpu_ms = (time.perf_counter() - t0) / reps * 1e3
    line = {
        "metric": "step modulations us per predict (AdaRMS rows of all layers and steps)", "value": ms * 1e3,
        "unit": "us", "higher_is_better": False, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) weights, U(-1,1) state)",
        "config": {"workload": f"{N} steps x MODW={MODW} modulation rows (projection {MODW}x{H} bf16)",
                   "N": N, "MODW": MODW, "l2": "256 MB written between timed steps (untimed); W_m 108.5 MB"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": f"{peak_kind} (hbm copy, burst)", "algorithmic_bytes": wbytes + io_bytes},
        "gpu_launches": 2 * args.steps,
        "clocks": clk,
        "cpu_baseline": {"value": cpu_ms * 1e3, "unit": "us", "cores": thr, "kind": "port",
                         "sample": f"{reps} full modulation computations, fp32 torch on the host"},
    }
    print(json.dumps(line), flush=True)


def run_prepare(args):
    """Cross-attention K/V preparation (register_prepare) of one predict, BASELINE configs[2]'s
    prepare part: all layers' K/V from S source rows x 2048, one tcgen05 GEMM launch. Prints one
    JSON line (not the headline metric)."""
    from reki_megakernel_b200.prepare import RegisterPrepare
    from reki_megakernel_b200.synthetic import ExpertDims, make_prepare_weights, make_source, rope_cos_sin
    dims = ExpertDims()
    pw = make_prepare_weights(dims, seed=0)
    src_h = make_source(args.S, dims.src_dim, seed=0)
    rp = RegisterPrepare(pw.to("cuda"))
    src = src_h.to("cuda")
    k, v = rp.run(src)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        rp.run(src, out=(k, v))
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        rp.run(src, out=(k, v))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    rp.check_device_error()
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.3)
    per = []
    for _ in range(args.steps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        per.append(a.elapsed_time(b))
    clk = clocks.stop()
    rp.check_device_error()
    ms = statistics.mean(per)
    L, H, D, S = dims.L, dims.H, dims.src_dim, args.S
    wbytes = L * 2 * H * D * 2
    io_bytes = S * D * 2 + 2 * L * S * H * 2 + L * dims.HD * 4 + 2 * S * dims.HD * 4
    flops = 2.0 * S * (L * 2 * H) * D
    hbm, peak_kind = peaks()
    achieved = (wbytes + io_bytes) / (ms * 1e-3) / 1e9
    # CPU: the same projection + norm/RoPE in fp32 on the host cores (the restatement, no float64)
    thr = len(os.sched_getaffinity(0))
    torch.set_num_threads(thr)
    c, sn = rope_cos_sin(torch.arange(S), dims.HD)
    x = src_h.float()
    wf = pw.wkv.float()
    t0 = time.perf_counter()
    reps = 0
    while reps < 2 or time.perf_counter() - t0 < 5.0:
        for l in range(L):
            kk = (x @ wf[l, 0].T).reshape(S, dims.NH, dims.HD)
            vv = x @ wf[l, 1].T
            kk = kk * torch.rsqrt(kk.pow(2).mean(-1, keepdim=True) + pw.eps) * (1.0 + pw.kn[l])
            rot = torch.cat([-kk[..., dims.HD // 2:], kk[..., :dims.HD // 2]], -1)
            kk = (kk * c[:, None] + rot * sn[:, None]).to(torch.bfloat16)
            vv = vv.to(torch.bfloat16)
        reps += 1
    cpu_ms = (time.perf_counter() - t0) / reps * 1e3
    line = {
        "metric": "register_prepare us per predict (cross-attention K/V of all layers)", "value": ms * 1e3,
        "unit": "us", "higher_is_better": False, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) projections, N(0,1)x0.5 source)",
        "config": {"workload": f"K/V projection of S={S} source rows x {D} for {L} layers + K head RMSNorm + RoPE",
                   "S": S, "src_dim": D, "layers": L, "l2": "256 MB written between timed steps (untimed)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": f"{peak_kind} (hbm copy, burst)", "algorithmic_bytes": wbytes + io_bytes},
        "tensor_tflops": flops / (ms * 1e-3) / 1e12,
        "gpu_launches": args.steps,
        "clocks": clk,
        "cpu_baseline": {"value": cpu_ms * 1e3, "unit": "us", "cores": thr, "kind": "port",
                         "sample": f"{reps} full preparations, fp32 torch on the host"},
    }
    print(json.dumps(line), flush=True)


def episodes_of_rank(rank: int, batch: int) -> list[int]:
    """Global episode indices served by this rank: ranks own disjoint, consecutive blocks of
    `batch` episodes, each seeded by its index."""
    return list(range(rank * batch, (rank + 1) * batch))


def max_over_ranks(vals, world: int, device) -> list[float]:
    """Element-wise max over ranks (the slowest rank bounds the job's time)."""
    t = torch.tensor([float(v) for v in vals], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(x) for x in t]


def job_episodes_per_s(world: int, batch: int, ms_per_step: float) -> float:
    """Whole-job throughput: every rank finishes `batch` episodes per step of `ms_per_step`."""
    return world * batch * 1000.0 / ms_per_step


def batch_algorithmic(dims, B: int, T: int, S: int, PM: int, SP: int, n_steps: int = 9):
    """(HBM bytes, FLOPs) one batched predict must move / compute: the weights and fp32 projections once
    per Euler step for all B episodes, and per episode and step its modulation row, register memory
    K/V (PM rows) and cross-attention K/V (S rows) of every layer; FLOPs of the dense stages
    (2 x rows x weights) and of the attention (scores and P V)."""
    L, H, I, A, HD = dims.L, dims.H, dims.I, dims.A, dims.HD
    wbytes = 2 * L * (3 * H * H + 3 * H * I + 3 * H * H) + 4 * 2 * A * H + 2 * 3 * L * HD
    per_ep = dims.MODW * 2 + L * (PM + S) * H * 2 * 2
    hbm = n_steps * (wbytes + B * per_ep)
    params = L * (3 * H * H + 3 * H * H + 3 * H * I)
    flops = n_steps * (2.0 * B * T * params + B * L * 4.0 * T * (PM + T + S) * H)
    return hbm, flops


def run_batch(args, rank: int, world: int):
    """B episodes per GPU through the batch path (BatchedExpert: one weight stream
    per Euler step for all of them, tcgen05 GEMMs over the stacked action rows). One step = one
    predict of all B episodes, replayed as a CUDA graph; value = episodes/s over the job."""
    from reki_megakernel_b200.batch import BatchedExpert
    from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_weights
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dims = ExpertDims()
    B = args.batch
    bx = BatchedExpert(make_weights(dims, seed=0).to(dev), max_episodes=B)
    # this rank's episodes rank * B .. rank * B + B - 1, each seeded by its global index
    host = make_inputs(dims, B=B, S=args.S, seed=1000 * rank * B, noise_seed=1234 + rank * B)
    inp = host.to(dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            bx.run(inp)
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = bx.run(inp)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    bx.check_device_error()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    t_wall = time.perf_counter()
    for a, b in evs:
        flush.fill_(1)
        a.record(stream)
        g.replay()
        b.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    wall = time.perf_counter() - t_wall
    clk = clocks.stop()
    bx.check_device_error()
    per = [a.elapsed_time(b) for a, b in evs]
    ms = statistics.mean(per)
    # end to end: every step copies all B episodes' inputs from pinned host memory, runs, reads back
    pinned = {k: (v.contiguous().pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in host.__dict__.items()}
    h2d = sum(v.numel() * v.element_size() for v in pinned.values() if isinstance(v, torch.Tensor))
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d2h = out_h.numel() * out_h.element_size()
    dev_t = {k: v for k, v in inp.__dict__.items() if isinstance(v, torch.Tensor)}

    def e2e_call():
        for k, v in dev_t.items():
            v.copy_(pinned[k], non_blocking=True)
        o = bx.run(inp)
        out_h.copy_(o, non_blocking=True)

    for _ in range(3):
        e2e_call()
    torch.cuda.synchronize(dev)
    e2e_ms = []
    for _ in range(max(5, args.steps // 4)):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        e2e_call()
        b.record(stream)
        b.synchronize()
        e2e_ms.append(a.elapsed_time(b))
    bx.check_device_error()
    ms_max, e2e_max = max_over_ranks([ms, statistics.mean(e2e_ms)], world, dev)
    if rank != 0:
        return
    PM, SP = host.memk.shape[2], host.kca.shape[2]
    hbm_bytes, flops = batch_algorithmic(dims, B, host.x.shape[1], args.S, PM - int(host.kv_start[0]), SP)
    hbm, peak_kind = peaks()
    tflops_peak = bf16_peak()
    achieved_gbs = hbm_bytes / (ms * 1e-3) / 1e9
    achieved_tf = flops / (ms * 1e-3) / 1e12
    tensor_bound = achieved_tf / tflops_peak[0] > achieved_gbs / hbm
    roof = ({"bound": "tensor", "achieved": achieved_tf, "peak": tflops_peak[0], "unit": "TFLOP/s",
             "frac": achieved_tf / tflops_peak[0], "peak_kind": tflops_peak[1]} if tensor_bound else
            {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s", "frac": achieved_gbs / hbm,
             "peak_kind": f"{peak_kind} (hbm copy, burst)"})
    roof.update({"traffic": None, "traffic_source": "not captured for the batch path",
                 "algorithmic_bytes_per_step": hbm_bytes, "flops_per_step": flops,
                 "hbm_gbs": achieved_gbs, "tflops": achieved_tf})
    line = {
        "metric": METRIC, "value": job_episodes_per_s(world, B, ms_max), "unit": "episodes/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "ms_per_predict": ms_max, "ms_per_step_p50": statistics.median(per),
        "ms_per_step_p99": sorted(per)[min(len(per) - 1, int(0.99 * len(per)))],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded weights, BASELINE configs[4] shapes, episodes seeded by index)",
        "config": dict(bench_config(args, world),
                       workload=f"REKI expert Euler steps 2-10 (BASELINE configs[4]): {B} episodes per GPU in one "
                                "batched predict (one weight stream, tcgen05 GEMMs over the stacked action rows)"),
        "roofline": roof,
        "e2e": {"value": job_episodes_per_s(world, B, e2e_max), "unit": "episodes/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_max},
        "gpu_launches": args.steps * bx.launches(B, host.x.shape[1], 9),
        "clocks": clk,
        "wall_s_timed_region": wall,
    }
    print(json.dumps(line), flush=True)


def bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "measured (cuBLAS bf16, burst)"
    return 1590.0, "fallback"


def run_mk(args, rank: int, world: int):
    from types import SimpleNamespace
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_past, make_weights
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dims = ExpertDims()
    w = make_weights(dims, seed=0)
    mk = ExpertMegakernel(weights=w.to(dev))
    del w
    # this rank's episodes, one batch-1 predict each per step (the kernel serves one episode per launch)
    eps = episodes_of_rank(rank, args.batch)
    inps = [make_inputs(dims, S=args.S, seed=e, noise_seed=1234 + e).to(dev) for e in eps]
    pasts = [make_past(i) for i in inps]

    def call():
        return [mk.run(i.x[:1], i.mods[0], i.dt[:1], pa, i.action_dim) for i, pa in zip(inps, pasts)]

    # CUDA graph of one step (steps 2..10 of every episode of this rank), as the expert graph holds it
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            call()
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = call()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    mk.check_device_error()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    t_wall = time.perf_counter()
    for a, b in evs:
        flush.fill_(1)              # L2 flush between timed steps (not timed)
        a.record(stream)
        g.replay()
        b.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    wall = time.perf_counter() - t_wall
    clk = clocks.stop()
    mk.check_device_error()
    per = [a.elapsed_time(b) for a, b in evs]
    ms = statistics.mean(per)
    # end to end through the public API: every step copies each episode's per-call inputs from
    # pinned host memory (ExpertMegakernel.run_from_host: the small inputs ahead of the launch, each
    # layer's K/V on a side stream under the first Euler step), launches, and reads each result back;
    # timed with events on the stream
    hosts, host_pasts = [], []
    for i, pa in zip(inps, pasts):
        rs = pa.register_step
        dev_in = {"x": i.x[:1], "mods": i.mods[0], "dt": i.dt[:1], "memk": i.memk[0], "memv": i.memv[0],
                  "kca": i.kca[0], "vca": i.vca[0], "cu_kv": rs["cu_kv"], "cu_src": rs["cu_src"],
                  "sa_cos": i.sa_cos[0], "sa_sin": i.sa_sin[0], "ca_cos": i.ca_cos[0], "ca_sin": i.ca_sin[0]}
        h = {k: v.cpu().contiguous().pin_memory() for k, v in dev_in.items()}
        hosts.append(h)
        host_pasts.append(SimpleNamespace(
            register_step={"mem_kv": [(h["memk"][l], h["memv"][l]) for l in range(dims.L)],
                           "sa_pe": (h["sa_cos"], h["sa_sin"]), "ca_pe": (h["ca_cos"], h["ca_sin"]),
                           "cu_kv": h["cu_kv"], "cu_src": h["cu_src"]},
            cross_attn_kv=[(h["kca"][l], h["vca"][l]) for l in range(dims.L)]))
    out_hosts = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    d2h = sum(o.numel() * o.element_size() for o in out_hosts)
    copied = []  # bytes each call of the last step copied in (the K/V rows the launch reads + small inputs)

    def e2e_call():
        copied.clear()
        for h, hp, i, oh in zip(hosts, host_pasts, inps, out_hosts):
            o = mk.run_from_host(h["x"], h["mods"], h["dt"], hp, i.action_dim)
            copied.append(mk.last_h2d_bytes)
            oh.copy_(o, non_blocking=True)

    for _ in range(max(3, args.warmup // 4)):
        e2e_call()
    torch.cuda.synchronize(dev)
    n_e2e = max(10, args.steps // 4)
    e2e_ms = []
    for _ in range(n_e2e):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        e2e_call()
        b.record(stream)
        b.synchronize()
        e2e_ms.append(a.elapsed_time(b))
    mk.check_device_error()
    e2e_mean = statistics.mean(e2e_ms)
    h2d = sum(copied)

    ms_max, e2e_max = max_over_ranks([ms, e2e_mean], world, dev)
    if rank != 0:
        return
    hbm, peak_kind = peaks()
    mods_row = dims.MODW * 2
    bytes_step = algorithmic_bytes_per_step(dims, mods_row)
    traffic, traffic_src = traffic_from_profile()
    # one launch streams the weights once: per-launch bytes over per-launch time
    achieved = 9 * bytes_step / (ms / args.batch * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": job_episodes_per_s(world, args.batch, ms_max), "unit": "episodes/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "ms_per_predict": ms_max / args.batch,
        "ms_per_step_p50": statistics.median(per), "ms_per_step_p99": sorted(per)[min(len(per) - 1, int(0.99 * len(per)))],
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": job_episodes_per_s(world, args.batch, ms_max) / (1000.0 / PUBLISHED_MS),
        "dtype": "bf16", "data": "synthetic (seeded weights, BASELINE configs[1] shapes)",
        "config": bench_config(args, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": f"{peak_kind} (hbm copy, burst)",
                     "traffic": traffic if args.S == 160 and args.batch == 1 else None,
                     "traffic_source": traffic_src, "algorithmic_bytes_per_launch": 9 * bytes_step},
        "e2e": {"value": job_episodes_per_s(world, args.batch, e2e_max), "unit": "episodes/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_max},
        "gpu_launches": args.steps * args.batch,
        "clocks": clk,
        "wall_s_timed_region": wall,
    }
    if world == 1 and not args.no_cpu_baseline:
        thr = len(os.sched_getaffinity(0))
        times = cpu_predict_ms(dims, args.S, thr, 1, 3, args.cpu_seconds)
        cpu_ms = statistics.median(times)
        line["cpu_baseline"] = {"value": 1000.0 / cpu_ms, "unit": "episodes/s", "cores": thr, "kind": "port",
                                "sample": f"{len(times)} whole predicts (9 Euler steps each) of one episode, fp32 CPU "
                                          "oracle, median", "ms_per_predict": cpu_ms}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="mk", choices=["mk", "reference"])
    ap.add_argument("--batch", type=int, default=1,
                    help="episodes per GPU; > 1 runs the batch path (one weight stream for all of them)")
    ap.add_argument("--S", type=int, default=160, help="cross-attention source rows (BASELINE configs[3]: 128-1024)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--max-ref-steps", type=int, default=60)
    ap.add_argument("--timeline", action="store_true", help="per-stage critical path of one predict, no bench line")
    ap.add_argument("--substage", action="store_true",
                    help="sub-phases of each stage from the traced profiling build, no bench line")
    ap.add_argument("--prepare", action="store_true", help="time register_prepare (cross-attention K/V), own JSON line")
    ap.add_argument("--mods", action="store_true", help="time the per-step modulation rows (_step_modulations), own JSON line")
    ap.add_argument("--predict", action="store_true",
                    help="time the GPU half of a predict after step 1 (modulations + K/V preparation + expert) as one graph")
    ap.add_argument("--full", action="store_true",
                    help="time whole carried predicts (all 10 steps, register pass, frame carry) as one graph each")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.timeline or args.substage or args.prepare or args.mods or args.predict or args.full:
        if rank == 0:
            (run_timeline if args.timeline else run_substage if args.substage else run_prepare if args.prepare
             else run_mods if args.mods else run_full if args.full else run_predict)(args)
        return
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if args.impl == "mk" else "gloo"
        kw = {}
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        torch.distributed.init_process_group(backend, timeout=timedelta(seconds=120), **kw)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.batch > 1:
            run_batch(args, rank, world)
        else:
            run_mk(args, rank, world)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
