"""Benchmark of the B200 MoE expert-FFN layer: MoE-layer tokens/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 4] [--tokens T] [--no-cpu-baseline] [--no-sweep]

Prints ONE JSON line on rank 0.

Workload (N=1 headline): configuration 4 of the benchmark, the largest
configuration that fits one B200 -- H=7168, 256 routed experts, top-8, one
always-on shared expert, I=2048, SwiGLU, MXFP4 weights (6.0 GB), 16,384
tokens per step.  Synthetic, seeded inputs (there is no dataset for this
path).  A step is one layer forward over one batch: router top-k,
permutation, quantise-once of the token rows, gate/up grouped GEMM + SwiGLU,
down grouped GEMM, weighted combine.

* value     tokens/s with inputs resident in HBM, timed with CUDA events on
            the launching stream (max over ranks).  The K timed steps are
            one window; the window is repeated until the timed work spans
            about three seconds (so the clock sampler sees the load), and
            the median window is reported;
* e2e       the same metric through the host-buffer C-ABI call
            (moe_b200_layer_forward_host): pinned-host x in, y/ids/weights out,
            copies inside the timed region;
* roofline  the dominant kernel, the gate/up grouped GEMM.  At prefill sizes
            (configs 2 to 4) it is tensor-bound: its algorithmic FLOPs per
            launch (4 H I per permuted row, the bf16-equivalent product the
            layer defines) over its CUDA-event duration, against the dense
            MXFP4 peak the metric names (9 PFLOP/s, spec); `issued` gives
            the same kernel against the rate of the MMA kind it issues
            (kind::mxf8f6f4, 4.5 PFLOP/s spec, two terms per product).
            MEASURED_PEAKS.json has no FP4 or FP8 figure, so both peaks are
            the spec's.  At decode sizes (config 0, 1) it is HBM-bound:
            algorithmic bytes against the measured HBM copy bandwidth;
* decode_sweep  the config 1 decode batches (1, 8, 32, 128, 256 tokens per
            step) on the same GPU, each with its whole-layer HBM fraction;
* cpu_baseline  the reference's own CPU path (oracle/_ref/libmoe_ref.so, the
            reference sources compiled by oracle/Makefile) timed on this host's
            cores over a prefix of the batch (kind "reference"), or the C
            restatement when that library is absent (kind "port").

L2: no flush between steps; instead the weights a step reads are never
still cached when they are read again.  At the headline workload one step
reads all 6.0 GB of the layer's weights against the 126 MB L2.  Where one
step's touched weights are smaller (config 0, small token counts, a rank's
expert block at 4 or 8 GPUs), the layer is uploaded into several layer
slots -- as a model's consecutive MoE layers would be -- and the steps cycle
through them, so that at least twice the L2 is read between two uses of one
copy (reported under "l2_reuse").

Multi-GPU (torchrun, N ranks): expert parallelism.  Experts are placed over
the ranks from a separate calibration batch (hot experts replicated), each
rank has its own batch of `--tokens` tokens (weak scaling); each step is
moe_b200_ep_layer_forward on every rank: local router, a device-side count
exchange, the assignment rows stored into their experts' owners over NVLink,
the local block-scaled expert GEMMs whose down-projection epilogue stores the
rows back to their source ranks, device barriers, and the combine.  value
sums the ranks' tokens over the slowest rank's CUDA-event time; the line also
reports the exchange's load balance (max / mean rows received per rank) and
a per-phase breakdown on rank 0.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "storage.llm_b200"
DEFAULT_CONFIG = 4
METRIC = "MoE-layer tokens/sec"


def load_pkg():
    if "moe_b200" in sys.modules:
        return sys.modules["moe_b200"]
    spec = importlib.util.spec_from_file_location("moe_b200", PKG / "__init__.py",
                                                  submodule_search_locations=[str(PKG)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moe_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# Dense tensor peaks from the B200 spec (TFLOP/s).  MEASURED_PEAKS.json has
# only bf16 (cuBLAS) and HBM figures.
MXFP4_TFLOPS = 9000.0     # kind::mxf4 (E2M1 x E2M1), the metric's roofline
MXF8F6F4_TFLOPS = 4500.0  # kind::mxf8f6f4 (the FP8 rate), the kind the GEMMs issue
L2_BYTES = 126e6    # B200 L2
MAX_COPIES = 16     # layer slots the engines are created with
WINDOW_SECONDS = 3.0
MAX_WINDOWS = 25


def expert_bytes(shape) -> float:
    """MXFP4 bytes of one expert triplet (17 bytes per 32 weights)."""
    return 3 * shape.intermediate * shape.hidden * 17 / 32


def weight_copies(touched_bytes: float) -> int:
    """Layer copies the timed steps cycle through so that at least twice the
    L2 is read between two uses of one copy's weights."""
    return int(max(1, min(MAX_COPIES, math.ceil(2 * L2_BYTES / max(touched_bytes, 1.0)))))


def default_tokens(synth, config: int) -> int:
    shape = synth.CONFIGS[config]
    return 256 if config == 1 else (shape.tokens or sum(synth.prefill_lengths()))


def is_prefill(config: int) -> bool:
    """Configurations whose GEMMs are tensor-bound (the metric's MXFP4
    roofline); decode-sized ones are HBM-bound."""
    return config >= 2


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons, power = [], 0.0, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        # samples under load: power at least half the peak seen (the sampler
        # starts just before the timed windows and stops just after them)
        pmax = max(power) if power else 0.0
        load = [s for s, p in zip(sm, power) if p >= 0.5 * pmax] or sm
        return {"sm_mhz": float(np.median(load)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "samples_under_load": len(load), "power_w_max": pmax}


# tokens of a batch the CPU arms time, per configuration: the reference runs
# the layer token by token, so the rate over a prefix is the batch's rate;
# the prefix keeps one CPU step near half a second on a 16-core host
CPU_SAMPLE_TOKENS = {0: 64, 1: 256, 2: 256, 3: 256, 4: 64}


def cpu_sample(li, config: int):
    """The prefix of a batch the CPU arms run, and the batch size."""
    T_all = li.x.shape[0]
    n = CPU_SAMPLE_TOKENS.get(config, 256)
    if T_all > n:
        li.x = np.ascontiguousarray(li.x[:n])
    return li, T_all


def cpu_runner(li, shape):
    """(run, kind, cores): the reference's CPU layer, or the C restatement."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # test infrastructure: the timed CPU baseline and reference arm only
    if oracle.REF_SO.exists():
        ref = oracle.Ref(oracle.metadata_json(shape.top_k, norm_topk=shape.norm_topk))
        return (lambda: ref.moe_layer(li)), "reference", int(ref.lib.ref_row_threads())
    if not oracle.PORT_SO.exists():
        oracle.build(ref=False)
    port = oracle.Port()
    cores = os.cpu_count() or 1
    return (lambda: port.moe_layer(li, threads=cores)), "port", cores


def host_cpu() -> str:
    try:
        return subprocess.run(["bash", "-c", "lscpu | grep 'Model name' | head -1 | cut -d: -f2"],
                              capture_output=True, text=True).stdout.strip()
    except OSError:
        return ""


def sample_text(reps, T, T_all, el=None):
    s = f"{reps} x {T}-token batches of the same workload" + (f" ({el:.1f} s)" if el is not None else "")
    if T < T_all:
        s += f", the first {T} of the step's {T_all} tokens (rate extrapolated)"
    return s + f", per-token reference layer order, -march=x86-64-v3, host CPU {host_cpu()}"


def cpu_baseline(li, shape, config: int, seconds: float = 12.0):
    """The reference's CPU layer (or the C restatement) on this host's cores."""
    li, T_all = cpu_sample(li, config)
    run, kind, cores = cpu_runner(li, shape)
    run()  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        run()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 40:
            break
    T = li.x.shape[0]
    return {"value": T * reps / el, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": sample_text(reps, T, T_all, el)}


def config_dict(shape, args):
    """The workload; identical in both arms (the GPU arm's L2 details are
    reported beside it, under l2_reuse)."""
    return {"workload": f"config{args.config}: H{shape.hidden} E{shape.experts} top{shape.top_k} "
                        f"I{shape.intermediate} SwiGLU MXFP4"
                        + (" + shared expert" if shape.shared else "")
                        + f", {args.tokens} tokens/step" + (f", skew {shape.skew}" if shape.skew else ""),
            "hidden": shape.hidden, "experts": shape.experts, "top_k": shape.top_k,
            "intermediate": shape.intermediate, "tokens_per_step": args.tokens, "shared_expert": shape.shared,
            "parallelism": f"ep{args.gpus}" if args.gpus > 1 else "single",
            "l2": "inputs_exceed_l2"}


def run_reference(args, shape, metric):
    """--impl reference: the reference's CPU path on the host cores."""
    import moe_b200.synth as synth
    li, T_all = cpu_sample(synth.make_layer(shape, seed=0, tokens=args.tokens), args.config)
    T = li.x.shape[0]
    step, kind, cores = cpu_runner(li, shape)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = T * args.steps / el
    return {"metric": metric, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": config_dict(shape, args),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                             "sample": sample_text(args.steps, T, T_all)},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def profiled_traffic(config: int, tokens: int):
    """DRAM bytes (read + write) per launch of the gate/up GEMM, from the ncu
    capture summarised under profiles/ for this workload (None without one).
    The summary names the workload it applies to on a `workload:` line."""
    for f in sorted((ROOT / "profiles").glob("gemm_bs_gate_up_c*.md")):
        txt = f.read_text().splitlines()
        wl = next((l.split(":", 1)[1].strip() for l in txt if l.startswith("workload:")), None)
        if wl != f"config{config} T={tokens}":
            continue
        for line in txt:
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    return None


class StdoutToStderr:
    """Points file descriptor 1 at stderr for the block: NCCL prints its
    version line to stdout when a communicator starts, and stdout carries
    only the one JSON line."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *a):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


def windows_for(step_s: float, steps: int) -> int:
    """Repetitions of the K-step window so the timed work spans about
    WINDOW_SECONDS."""
    return int(max(1, min(MAX_WINDOWS, math.ceil(WINDOW_SECONDS / max(step_s * steps, 1e-6)))))


def timed_windows(step, steps, windows, stream, dist=None):
    """`windows` windows of exactly `steps` steps, each bracketed by a barrier
    (multi-GPU) and device synchronisation on both sides and timed with CUDA
    events on the launching stream; returns the per-window milliseconds
    (max over ranks)."""
    import torch
    out = []
    for _ in range(windows):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
        ms = start.elapsed_time(end)
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        out.append(ms)
    return out


def warmup_step_seconds(step, warmup, dist=None):
    """Runs the warm-up steps; returns the seconds per step of the last half
    (agreed over ranks, so every rank times the same number of windows)."""
    import torch
    half = max(1, warmup // 2)
    for _ in range(warmup - half):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(half):
        step()
    torch.cuda.synchronize()
    s = (time.perf_counter() - t0) / half
    if dist:
        t = torch.tensor([s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        s = float(t.item())
    return s


def calibrate_placement(shape, li, rank, world, dist, tokens):
    """Expert placement with replication from a calibration batch (not the
    timed tokens): per-expert routing counts summed over the ranks, experts
    whose load exceeds a rank's share split into replicas, replicas placed
    largest first on the least-loaded rank not yet holding that expert.
    Every rank computes the same placement from the same counts."""
    import torch
    import moe_b200.synth as synth
    xc = synth.gen_tokens(shape, min(tokens, 4096), seed=900 + rank, mu=li.mu)
    xf = (xc.astype(np.uint32) << 16).view(np.float32)
    wf = (np.ascontiguousarray(li.router).astype(np.uint32) << 16).view(np.float32)
    logits = xf @ wf.T  # routing decisions only; the layer itself routes exactly
    top = np.argsort(-logits, axis=1, kind="stable")[:, :shape.top_k]
    counts = torch.tensor(np.bincount(top.ravel(), minlength=shape.experts).astype(np.float64), device="cuda")
    dist.all_reduce(counts)
    return place_replicas(counts.cpu().numpy(), world)


def place_replicas(counts, world):
    """Replica placement from per-expert routing counts: an expert whose load
    exceeds one rank's share gets that many replicas (at most `world`), each
    carrying an equal part of its load; replicas go largest first to the
    least-loaded rank not yet holding that expert (lower rank on ties).
    Returns (replica ranks per expert, planned max / mean rank load)."""
    E = len(counts)
    share = float(np.sum(counts)) / world
    reps = [int(min(world, max(1, np.ceil(c / max(share, 1.0))))) for c in counts]
    items = sorted(((counts[e] / reps[e], e) for e in range(E) for _ in range(reps[e])), key=lambda t: (-t[0], t[1]))
    load = np.zeros(world)
    placement = [[] for _ in range(E)]
    for w_, e in items:
        order = sorted(range(world), key=lambda q: (load[q], q))
        q = next(q for q in order if q not in placement[e])
        placement[e].append(q)
        load[q] += w_
    return placement, (load.max() / max(load.mean(), 1e-9))


def layer_flops(shape, T):
    """Algorithmic FLOPs of one layer call (bf16-equivalent products):
    T k 6 H I (+ T 6 H I shared) + 2 T H E (router)."""
    H, I, E, K = shape.hidden, shape.intermediate, shape.experts, shape.top_k
    return T * (K + (1 if shape.shared else 0)) * 6 * H * I + 2 * T * H * E


def layer_bytes(shape, T, distinct):
    """Algorithmic HBM bytes of one layer call: the MXFP4 weights of the
    distinct experts routed to (+ the shared expert), the router rows, the
    token rows in and out, and the permuted rows written and read once."""
    H, E, K = shape.hidden, shape.experts, shape.top_k
    wts = (distinct + (1 if shape.shared else 0)) * expert_bytes(shape)
    return wts + E * H * 2 + 2 * T * H * 2 + 2 * T * K * H * 2


def tensor_roofline(shape, T, gu_ms, dn_ms, traffic, fp4=False):
    """The gate/up GEMM against the metric's MXFP4 roofline, and against the
    rate of the MMA kind it issues: two E4M3 terms per bf16 activation at the
    FP8 rate, or (fast mode) one E2M1 term at the MXFP4 rate."""
    H, I = shape.hidden, shape.intermediate
    P = T * (shape.top_k + (1 if shape.shared else 0))
    gu_flops = P * 4.0 * H * I
    dn_flops = P * 2.0 * H * I
    ach = gu_flops / (gu_ms / 1e3) / 1e12
    dn_ach = dn_flops / (dn_ms / 1e3) / 1e12
    _, bf16, bf16_kind = measured_peaks()
    return {"kernel": "gemm_bs_kernel<gate_up> (grouped MXFP4 gate/up GEMM + SwiGLU)", "bound": "tensor",
            "achieved": ach, "peak": MXFP4_TFLOPS, "unit": "TFLOP/s", "frac": ach / MXFP4_TFLOPS,
            "peak_source": "spec: dense MXFP4 9 PFLOP/s (MEASURED_PEAKS.json has no FP4 or FP8 figure)",
            "traffic": traffic, "algorithmic_flops_per_launch": gu_flops, "launch_ms": gu_ms,
            "issued": ({"mma": "tcgen05.mma kind::mxf4 block_scale: E2M1 weights x E2M1 activations",
                        "flops_issued_per_launch": gu_flops, "achieved": ach, "peak": MXFP4_TFLOPS,
                        "frac": ach / MXFP4_TFLOPS, "peak_source": "spec: dense MXFP4 9 PFLOP/s"} if fp4 else
                       {"mma": "tcgen05.mma kind::mxf8f6f4 block_scale: E2M1 weights x E4M3 hi + lo activation terms",
                        "flops_issued_per_launch": 2 * gu_flops, "achieved": 2 * ach, "peak": MXF8F6F4_TFLOPS,
                        "frac": 2 * ach / MXF8F6F4_TFLOPS, "peak_source": "spec: dense FP8-rate 4.5 PFLOP/s"}),
            "vs_measured_bf16_cublas": {"peak": bf16, "frac": ach / bf16, "peak_source": bf16_kind},
            "down_gemm": {"achieved": dn_ach, "unit": "TFLOP/s", "launch_ms": dn_ms, "frac": dn_ach / MXFP4_TFLOPS,
                          "issued_frac": dn_ach / MXFP4_TFLOPS if fp4 else 2 * dn_ach / MXF8F6F4_TFLOPS}}


def run_expert_parallel(args, shape, li, metric, rank, world, local, dist):
    """--gpus N > 1: moe_b200_ep_layer_forward on every rank (see the module docstring)."""
    import ctypes as C
    import torch
    import moe_b200.lib as L

    T, H, K = args.tokens, shape.hidden, shape.top_k
    eng = L.Engine(local, max_layers=MAX_COPIES)
    with StdoutToStderr():
        uid = [L.Engine.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eng.ep_init(rank, world, uid[0])
        dist.barrier()
    placement, planned_imbalance = calibrate_placement(shape, li, rank, world, dist, T)
    eng.ep_set_placement(placement)
    # copies of the layer to cycle through, from the smallest expert block
    # any rank holds (the placement is the same on every rank, so is this)
    min_block = min(sum(q in reps for reps in placement) for q in range(world))
    touched = (min_block + (1 if shape.shared else 0)) * expert_bytes(shape)
    copies = weight_copies(touched)
    for layer in range(copies):
        eng.upload_layer_ep(li, layer=layer)
    li.gate = li.up = li.down = None  # the host copies of the weights are no longer needed
    cfgs = [L.Engine.cfg(shape, layer=layer, gemm_path=L.GEMM_BLOCKSCALED) for layer in range(copies)]
    calls = [0]

    def next_cfg():
        calls[0] += 1
        return cfgs[(calls[0] - 1) % copies]

    x = torch.from_numpy(li.x.view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.int16, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step():
        eng.ep_forward(next_cfg(), x, T, y_bf16=y, ids=ids, w=w, stream=sp)

    step_s = warmup_step_seconds(step, args.warmup, dist)
    eng.sync(sp)
    launches_per_step = eng.launches()
    windows = args.windows or windows_for(step_s, args.steps)
    dist.barrier()
    with ClockSampler(local) as clk:
        win_ms = timed_windows(step, args.steps, windows, stream, dist)
    eng.sync(sp)
    ms = float(np.median(win_ms))
    dist.barrier()
    value = T * args.steps * world / (ms / 1000.0)
    # per-phase breakdown: the same steps again with events between phases
    eng.profile_enable(args.steps)
    for _ in range(args.steps):
        step()
    eng.sync(sp)
    phase_ms, prof_calls = eng.profile_read()
    eng.profile_enable(0)
    ep_phases = dict(zip(("router", "dispatch", "counts_sync", "row_exchange", "local_experts",
                          "return_combine"), [v / max(prof_calls, 1) for v in phase_ms.values()]))
    sent, recv = eng.ep_last_counts(world)
    rows = torch.tensor([float(recv.sum())], device="cuda")
    rows_all = [torch.zeros_like(rows) for _ in range(world)]
    dist.all_gather(rows_all, rows)
    rows_all = [float(r.item()) for r in rows_all]
    imbalance = max(rows_all) / max(np.mean(rows_all), 1e-9)

    # end to end through the host-pointer C-ABI call
    xh = torch.from_numpy(li.x.view(np.int16)).pin_memory()
    yh = torch.empty((T, H), dtype=torch.int16).pin_memory()
    idsh = torch.empty((T, K), dtype=torch.int32).pin_memory()
    wh = torch.empty((T, K), dtype=torch.float32).pin_memory()
    lib = L.load()

    def step_host():
        ok = lib.moe_b200_ep_layer_forward_host(eng.h, C.byref(next_cfg()), xh.data_ptr(), T, yh.data_ptr(),
                                                None, idsh.data_ptr(), wh.data_ptr(), eng.err)
        if not ok:
            raise L.MoEError(eng.err.value.decode())

    for _ in range(3):
        step_host()
    dist.barrier()
    torch.cuda.synchronize()
    n_e2e = torch.tensor([args.e2e_steps or max(args.steps, int(math.ceil(2.0 / max(step_s, 1e-6))))],
                         device="cuda")
    dist.all_reduce(n_e2e, op=dist.ReduceOp.MAX)
    e2e_steps = int(n_e2e.item())
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_host()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = T * e2e_steps * world / float(t.item())

    e_loc = len(eng.ep_local_expert_list(shape.experts))
    step_ms = ms / args.steps
    if is_prefill(args.config):
        # one rank's expert GEMMs: every row it received plus its own shared rows
        P = float(recv.sum()) + (T if shape.shared else 0)
        flops = P * 6.0 * H * shape.intermediate
        ach = flops / (step_ms / 1e3) / 1e12
        roofline = {"kernel": "whole layer on one expert-parallel rank (its grouped GEMMs' FLOPs over the step)",
                    "bound": "tensor", "achieved": ach, "peak": MXFP4_TFLOPS, "unit": "TFLOP/s",
                    "frac": ach / MXFP4_TFLOPS,
                    "peak_source": "spec: dense MXFP4 9 PFLOP/s (MEASURED_PEAKS.json has no FP4 or FP8 figure)",
                    "traffic": None, "algorithmic_flops_per_launch": flops, "launch_ms": step_ms,
                    "issued": {"achieved": 2 * ach, "peak": MXF8F6F4_TFLOPS, "frac": 2 * ach / MXF8F6F4_TFLOPS}}
    else:
        hbm, _, peak_kind = measured_peaks()
        lb = e_loc * expert_bytes(shape) + T * H * 2 * 2 + 2 * T * K * H * 2
        achieved = lb / (step_ms / 1000.0) / 1e9
        roofline = {"kernel": "whole layer on one expert-parallel rank", "bound": "hbm", "achieved": achieved,
                    "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "peak_source": peak_kind,
                    "traffic": None, "algorithmic_bytes_per_launch": lb, "launch_ms": step_ms}
    result = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": config_dict(shape, args),
        "l2_reuse": {"weight_copies_cycled": copies, "weight_bytes_between_reuses": touched * copies},
        "timing": {"windows": windows, "window_ms": win_ms, "reported": "median window"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2 * world,
                "d2h_bytes_per_step": (T * H * 2 + T * K * 8) * world, "steps": e2e_steps},
        "roofline": roofline,
        "expert_parallel": {"experts_per_gpu": e_loc, "rows_received_per_rank": rows_all,
                            "placement": "replicated, calibrated on a separate batch",
                            "replicas_per_expert": [len(r) for r in placement],
                            "planned_imbalance": planned_imbalance,
                            "load_imbalance_max_over_mean": imbalance, "phase_ms_rank0": ep_phases},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(result), flush=True)
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


def single_gpu_layer(args, shape, li, local, eng, L, uploaded, sample_clocks=True, gemm_path=0):
    """One configuration on one GPU: value, stages and e2e.  `uploaded` is
    the set of layer slots of `eng` that already hold this layer (slot 0 at
    least); more copies are uploaded when a step touches little."""
    import ctypes as C
    import torch

    T, H, K = li.x.shape[0], shape.hidden, shape.top_k
    cfg = L.Engine.cfg(shape, gemm_path=gemm_path)
    x = torch.from_numpy(li.x.view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.int16, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    # one call tells which experts the batch routes to, hence the weight
    # bytes a step reads and how many copies of the layer to cycle through
    eng.forward(cfg, x, T, y_bf16=y, ids=ids, w=w, stream=sp)
    eng.sync(sp)
    routed = int((eng.read(L.BUF_GROUP_COUNT, (shape.experts,), np.uint32) > 0).sum())
    touched = (routed + (1 if shape.shared else 0)) * expert_bytes(shape)
    copies = weight_copies(touched)
    for layer in range(1, copies):
        if layer not in uploaded:
            eng.upload_layer(li, layer=layer)
            uploaded.add(layer)
    cfgs = [cfg] + [L.Engine.cfg(shape, layer=layer, gemm_path=gemm_path) for layer in range(1, copies)]
    calls = [0]

    def next_cfg():
        calls[0] += 1
        return cfgs[(calls[0] - 1) % copies]

    def step():
        eng.forward(next_cfg(), x, T, y_bf16=y, ids=ids, w=w, stream=sp)

    step_s = warmup_step_seconds(step, args.warmup)
    eng.sync(sp)
    launches_per_step = eng.launches()
    windows = args.windows or windows_for(step_s, args.steps)
    clk = None
    if sample_clocks:
        with ClockSampler(local) as clk:
            win_ms = timed_windows(step, args.steps, windows, stream)
    else:
        win_ms = timed_windows(step, args.steps, windows, stream)
    eng.sync(sp)
    ms = float(np.median(win_ms))
    value = T * args.steps / (ms / 1000.0)

    # per-stage breakdown: the same steps again with events between the
    # stages (kept out of the headline region above)
    eng.profile_enable(args.steps)
    for _ in range(args.steps):
        step()
    eng.sync(sp)
    stage_ms, prof_calls = eng.profile_read()
    eng.profile_enable(0)
    stages = {k: v / max(prof_calls, 1) for k, v in stage_ms.items()}

    # end to end through the host-buffer C-ABI call
    xh = torch.from_numpy(li.x.view(np.int16)).pin_memory()
    yh = torch.empty((T, H), dtype=torch.int16).pin_memory()
    idsh = torch.empty((T, K), dtype=torch.int32).pin_memory()
    wh = torch.empty((T, K), dtype=torch.float32).pin_memory()
    lib = L.load()

    def step_host():
        ok = lib.moe_b200_layer_forward_host(eng.h, C.byref(next_cfg()), xh.data_ptr(), T, yh.data_ptr(), None,
                                             idsh.data_ptr(), wh.data_ptr(), None, eng.err)
        if not ok:
            raise L.MoEError(eng.err.value.decode())

    for _ in range(3):
        step_host()
    torch.cuda.synchronize()
    e2e_steps = args.e2e_steps or max(args.steps, int(math.ceil(2.0 / max(step_s, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_host()
    torch.cuda.synchronize()
    e2e_value = T * e2e_steps / (time.perf_counter() - t0)

    counts = eng.read(L.BUF_GROUP_COUNT, (shape.experts,), np.uint32)
    distinct = int((counts > 0).sum())
    return dict(value=value, ms=ms, win_ms=win_ms, windows=windows, stages=stages, e2e=e2e_value,
                e2e_steps=e2e_steps, distinct=distinct, copies=copies, touched=touched,
                launches=launches_per_step, clk=clk)


def fast_mode(args, shape, li, local, eng, L):
    """The opt-in fast mode (MOE_B200_GEMM_MXF4_FAST: E2M1 activations and
    intermediate, kind::mxf4 GEMMs) on the same workload: its throughput, its
    GEMMs against the MXFP4 roofline, and how far its output is from the
    tolerance-matched path's on a sample of the batch (it is not held to the
    layer tolerance)."""
    T = li.x.shape[0]
    r = single_gpu_layer(args, shape, li, local, eng, L, {0}, sample_clocks=False, gemm_path=L.GEMM_MXF4_FAST)
    sample = np.sort(np.random.default_rng(11).choice(T, size=min(64, T), replace=False))
    xs = np.ascontiguousarray(li.x[sample])
    exact = eng.forward_host(L.Engine.cfg(shape), xs)["y_f32"].astype(np.float64)
    fast = eng.forward_host(L.Engine.cfg(shape, gemm_path=L.GEMM_MXF4_FAST), xs)["y_f32"].astype(np.float64)
    d = np.abs(fast - exact)
    st = r["stages"]
    return {"gemm_path": "MOE_B200_GEMM_MXF4_FAST", "tolerance_matched": False,
            "value": r["value"], "unit": "tokens/s", "ms_per_step": r["ms"] / args.steps, "e2e": r["e2e"],
            "stages_ms_per_step": st,
            "roofline": tensor_roofline(shape, T, st["gate_up"], st["down"], None, fp4=True),
            "deviation_from_exact_path": {"tokens": int(len(sample)),
                                          "max_abs_over_max_abs_y": float(d.max() / np.abs(exact).max()),
                                          "mean_rel": float(d.mean() / np.abs(exact).mean())}}


def decode_sweep(args, local, L, synth):
    """Config 1 at each decode batch size of its sweep, with the whole-layer
    HBM fraction (algorithmic bytes / step time against the measured copy
    bandwidth)."""
    import torch
    shape = synth.CONFIGS[1]
    hbm, _, peak_kind = measured_peaks()
    eng = L.Engine(local, max_layers=MAX_COPIES)
    points = []
    try:
        li0 = synth.make_layer(shape, seed=0, tokens=256)
        eng.upload_layer(li0)
        uploaded = {0}
        for T in synth.DECODE_SWEEP:
            li = synth.LayerInputs(shape, li0.router, li0.gate, li0.up, li0.down,
                                   synth.gen_tokens(shape, T, 0, li0.mu), mu=li0.mu)
            r = single_gpu_layer(args, shape, li, local, eng, L, uploaded, sample_clocks=False)
            step_ms = r["ms"] / args.steps
            lb = layer_bytes(shape, T, r["distinct"])
            ach = lb / (step_ms / 1e3) / 1e9
            points.append({"tokens": T, "tokens_per_s": r["value"], "ms_per_step": step_ms,
                           "e2e_tokens_per_s": r["e2e"], "distinct_experts": r["distinct"],
                           "algorithmic_bytes": lb, "achieved_gbs": ach, "hbm_frac": ach / hbm,
                           "weight_copies_cycled": r["copies"], "stages_ms_per_step": r["stages"]})
        torch.cuda.synchronize()
    finally:
        eng.close()
    return {"workload": f"config1: H{shape.hidden} E{shape.experts} top{shape.top_k} I{shape.intermediate} "
                        f"SwiGLU MXFP4, skew {shape.skew}", "peak_gbs": hbm, "peak_source": peak_kind,
            "points": points}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=DEFAULT_CONFIG)
    ap.add_argument("--tokens", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config 1 decode sweep of the default line")
    ap.add_argument("--no-fast", action="store_true", help="skip the fast-mode (kind::mxf4) figures")
    # for profiling runs (a short, fixed launch sequence under ncu)
    ap.add_argument("--windows", type=int, default=0, help="timed windows (0: enough for ~3 s)")
    ap.add_argument("--e2e-steps", type=int, default=0, help="host-buffer steps (0: enough for ~2 s)")
    ap.add_argument("--gemm-path", default="exact", choices=["exact", "fast"],
                    help="profiling only: run the main line through the fast mode")
    ap.add_argument("--experts", type=int, default=0,
                    help="profiling only: the configuration's shapes with this many routed experts")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    load_pkg()
    import moe_b200.synth as synth

    shape = synth.CONFIGS[args.config]
    if args.experts:
        import dataclasses
        shape = dataclasses.replace(shape, name=f"{shape.name}_e{args.experts}", experts=args.experts)
    if args.tokens <= 0:
        args.tokens = default_tokens(synth, args.config)
    metric = METRIC

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, shape, metric)), flush=True)
        return

    import torch
    import moe_b200.lib as L

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))

    li = synth.make_layer(shape, seed=0, tokens=args.tokens)
    if world > 1:  # each rank its own token batch (weak scaling)
        li.x = synth.gen_tokens(shape, args.tokens, seed=100 + rank, mu=li.mu)
        run_expert_parallel(args, shape, li, metric, rank, world, local, dist)
        return
    eng = L.Engine(local, max_layers=MAX_COPIES)
    eng.upload_layer(li)
    main_path = L.GEMM_MXF4_FAST if args.gemm_path == "fast" else L.GEMM_BLOCKSCALED
    r = single_gpu_layer(args, shape, li, local, eng, L, {0}, gemm_path=main_path)
    T, H, K = args.tokens, shape.hidden, shape.top_k
    stages = r["stages"]
    gu_ms, dn_ms = stages["gate_up"], stages["down"]
    hbm, _, peak_kind = measured_peaks()
    P = T * K + (T if shape.shared else 0)
    if is_prefill(args.config):
        roofline = tensor_roofline(shape, T, gu_ms, dn_ms, profiled_traffic(args.config, T),
                                   fp4=main_path == L.GEMM_MXF4_FAST)
    else:
        # gate/up: the routed experts' gate and up weights + the permuted
        # rows in + the intermediate out, at 2 bytes per element
        gu_bytes = (r["distinct"] + (1 if shape.shared else 0)) * 2 * shape.intermediate * H * 17 / 32 \
            + P * H * 2 + P * shape.intermediate * 2
        achieved = gu_bytes / (gu_ms / 1000.0) / 1e9
        roofline = {"kernel": "gemm_bs_kernel<gate_up>", "bound": "hbm", "achieved": achieved, "peak": hbm,
                    "unit": "GB/s", "frac": achieved / hbm, "peak_source": peak_kind,
                    "traffic": profiled_traffic(args.config, T), "algorithmic_bytes_per_launch": gu_bytes,
                    "launch_ms": gu_ms, "distinct_experts": r["distinct"]}
    step_ms = r["ms"] / args.steps
    lf = layer_flops(shape, T)
    result = {
        "metric": metric, "value": r["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": config_dict(shape, args),
        "gemm_path": ("fast mode (kind::mxf4, not tolerance-matched)" if main_path == L.GEMM_MXF4_FAST
                      else "block-scaled, tolerance-matched"),
        "l2_reuse": {"weight_copies_cycled": r["copies"], "weight_bytes_between_reuses": r["touched"] * r["copies"]},
        "timing": {"windows": r["windows"], "window_ms": r["win_ms"], "reported": "median window"},
        "e2e": {"value": r["e2e"], "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2 + T * K * 8, "steps": r["e2e_steps"]},
        "roofline": roofline,
        "layer": {"algorithmic_flops": lf, "tflops": lf / (step_ms / 1e3) / 1e12,
                  "frac_of_mxfp4_peak": lf / (step_ms / 1e3) / 1e12 / MXFP4_TFLOPS,
                  "algorithmic_bytes": layer_bytes(shape, T, r["distinct"]),
                  "distinct_experts": r["distinct"]},
        "stages_ms_per_step": stages,
        "gpu_launches": r["launches"] * args.steps,
        "clocks": r["clk"].summary() if r["clk"] else None,
    }
    if is_prefill(args.config) and not args.no_fast:
        result["fast_mode"] = fast_mode(args, shape, li, local, eng, L)
    eng.close()
    if args.config == DEFAULT_CONFIG and not args.no_sweep:
        result["decode_sweep"] = decode_sweep(args, local, L, synth)
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(li, shape, args.config)
    print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
