"""Benchmark of the B200 MoE expert-FFN layer: MoE-layer tokens/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1] [--tokens 256]

Prints ONE JSON line on rank 0.

Workload (N=1 headline): configuration 1 of the benchmark -- H=2880, 32
experts, top-4, I=2880, SwiGLU, MXFP4 weights, Zipf(1.1)-skewed routing --
at its largest decode batch, 256 tokens per step.  Synthetic, seeded inputs
(there is no dataset for this path).  A step is one layer forward over one
batch: router top-k, permutation, gather, gate/up grouped GEMM + SwiGLU, down
grouped GEMM, weighted combine.

* value     tokens/s over the timed steps with inputs resident in HBM, timed
            with CUDA events on the launching stream (max over ranks);
* e2e       the same metric through the host-buffer C-ABI call
            (moe_b200_layer_forward_host): pinned-host x in, y/ids/weights out,
            copies inside the timed region;
* roofline  the dominant kernel (gate/up grouped GEMM): algorithmic bytes per
            launch (MXFP4 bytes of the distinct experts routed to + activation
            rows in + intermediate out) / its CUDA-event duration, against the
            measured HBM copy bandwidth;
* cpu_baseline  the reference's own CPU path (oracle/_ref/libmoe_ref.so, the
            reference sources compiled by oracle/Makefile) timed on this host's
            cores over one 256-token batch (kind "reference"), or the C
            restatement when that library is absent (kind "port").

L2: no flush between steps; instead the weights a step reads are never
still cached when they are read again.  At the headline workload one layer's
routed experts are 423 MB against the 126 MB L2.  Where one layer's touched
weights are smaller (config 0, small token counts, a rank's expert block at 4
or 8 GPUs), the layer is uploaded into several layer slots -- as a model's
consecutive MoE layers would be -- and the steps cycle through them, so that
at least twice the L2 is read between two uses of one copy
("weight_copies_cycled" in `config`).

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


L2_BYTES = 126e6    # B200 L2
MAX_COPIES = 16     # layer slots the engines are created with


def expert_bytes(shape) -> float:
    """MXFP4 bytes of one expert triplet (17 bytes per 32 weights)."""
    return 3 * shape.intermediate * shape.hidden * 17 / 32


def weight_copies(touched_bytes: float) -> int:
    """Layer copies the timed steps cycle through so that at least twice the
    L2 is read between two uses of one copy's weights."""
    return int(max(1, min(MAX_COPIES, math.ceil(2 * L2_BYTES / max(touched_bytes, 1.0)))))


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
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        load = sorted(sm)[len(sm) // 2:]  # upper half ~ under load
        return {"sm_mhz": float(np.median(load)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


CPU_SAMPLE_TOKENS = 256  # tokens per CPU-timed batch (the headline's whole batch)


def cpu_sample(li):
    """The first CPU_SAMPLE_TOKENS tokens of a batch, and the batch size.
    Each token goes through the reference layer on its own, so the rate over
    a prefix is the rate over the batch; larger batches (configs 2 to 4)
    are timed on their prefix so the CPU arms end within minutes."""
    T_all = li.x.shape[0]
    if T_all > CPU_SAMPLE_TOKENS:
        li.x = np.ascontiguousarray(li.x[:CPU_SAMPLE_TOKENS])
    return li, T_all


def cpu_baseline(li, seconds: float = 12.0):
    """The reference's CPU layer (or the C restatement) on this host's cores."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # test infrastructure: the timed CPU baseline only
    li, T_all = cpu_sample(li)
    s = li.shape
    if oracle.REF_SO.exists():
        ref = oracle.Ref(oracle.metadata_json(s.top_k, norm_topk=s.norm_topk))
        run = lambda: ref.moe_layer(li)
        kind, cores = "reference", int(ref.lib.ref_row_threads())
    else:
        if not oracle.PORT_SO.exists():
            oracle.build(ref=False)
        port = oracle.Port()
        cores = os.cpu_count() or 1
        run = lambda: port.moe_layer(li, threads=cores)
        kind = "port"
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
    try:
        cpu = subprocess.run(["bash", "-c", "lscpu | grep 'Model name' | head -1 | cut -d: -f2"],
                             capture_output=True, text=True).stdout.strip()
    except OSError:
        cpu = ""
    return {"value": T * reps / el, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{reps} x {T}-token batches of the same workload ({el:.1f} s)"
                      + (f", the first {T} of the step's {T_all} tokens (rate extrapolated)" if T < T_all else "")
                      + f", per-token reference layer order, -march=x86-64-v3, host CPU {cpu}"}


def run_reference(args, shape, metric):
    """--impl reference: the reference's CPU path on the host cores."""
    import moe_b200.synth as synth
    li, T_all = cpu_sample(synth.make_layer(shape, seed=0, tokens=args.tokens))
    T = li.x.shape[0]
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    if oracle.REF_SO.exists():
        ref = oracle.Ref(oracle.metadata_json(shape.top_k, norm_topk=shape.norm_topk))
        step = lambda: ref.moe_layer(li)
        kind, cores = "reference", int(ref.lib.ref_row_threads())
    else:
        if not oracle.PORT_SO.exists():
            oracle.build(ref=False)
        port = oracle.Port()
        cores = os.cpu_count() or 1
        step = lambda: port.moe_layer(li, threads=cores)
        kind = "port"
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
                             "sample": f"{args.steps} x {T}-token batches"
                                       + (f", the first {T} of the step's {T_all} tokens (rate extrapolated)"
                                          if T < T_all else "")},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def config_dict(shape, args, copies: int = 1, touched_bytes: float | None = None):
    d = {"workload": f"config{args.config}: H{shape.hidden} E{shape.experts} top{shape.top_k} "
                     f"I{shape.intermediate} SwiGLU MXFP4, {args.tokens} tokens/step"
                     + (f", skew {shape.skew}" if shape.skew else ""),
         "hidden": shape.hidden, "experts": shape.experts, "top_k": shape.top_k,
         "intermediate": shape.intermediate, "tokens_per_step": args.tokens, "shared_expert": shape.shared,
         "parallelism": f"ep{args.gpus}" if args.gpus > 1 else "single",
         "l2": "inputs_exceed_l2"}
    if touched_bytes is not None:  # the GPU arms: weights read between two uses of one copy
        d["weight_copies_cycled"] = copies
        d["weight_bytes_between_reuses"] = touched_bytes * copies
    return d


def profiled_traffic(args):
    """DRAM bytes (read + write) per launch of the gate/up GEMM, from the ncu
    capture summarised under profiles/ for this workload (None without one)."""
    if args.config != 1 or args.tokens != 256:
        return None
    f = ROOT / "profiles" / "gemm_bs_gate_up_c1_t256.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
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


def calibrate_placement(shape, li, rank, world, dist, tokens):
    """Expert placement with replication from a calibration batch (not the
    timed tokens): per-expert routing counts summed over the ranks, experts
    whose load exceeds a rank's share split into replicas, replicas placed
    largest first on the least-loaded rank not yet holding that expert.
    Every rank computes the same placement from the same counts."""
    import torch
    import moe_b200.synth as synth
    xc = synth.gen_tokens(shape, tokens, seed=900 + rank, mu=li.mu)
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

    for _ in range(args.warmup):
        step()
    eng.sync(sp)
    launches_per_step = eng.launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
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

    for _ in range(10):
        step_host()
    dist.barrier()
    torch.cuda.synchronize()
    e2e_steps = max(200, args.steps)  # host wall clock: a longer window for a steadier figure
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_host()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = T * e2e_steps * world / float(t.item())

    # whole-layer HBM roofline of one rank: its expert block's MXFP4 bytes
    # (every local expert is routed to at these batch sizes) + its token rows
    hbm, _, peak_kind = measured_peaks()
    e_loc = len(eng.ep_local_expert_list(shape.experts))
    layer_bytes = e_loc * 3 * shape.intermediate * H * 17 / 32 + T * H * 2 * 2 + 2 * T * K * H * 2
    achieved = layer_bytes / (ms / args.steps / 1000.0) / 1e9
    result = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": config_dict(shape, args, copies, touched),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2 * world,
                "d2h_bytes_per_step": (T * H * 2 + T * K * 8) * world},
        "roofline": {"kernel": "whole layer on one expert-parallel rank", "bound": "hbm", "achieved": achieved,
                     "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "peak_source": peak_kind,
                     "traffic": None, "algorithmic_bytes_per_launch": layer_bytes,
                     "launch_ms": ms / args.steps},
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--tokens", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    load_pkg()
    import moe_b200.synth as synth

    shape = synth.CONFIGS[args.config]
    if args.tokens <= 0:
        args.tokens = 256 if args.config == 1 else (shape.tokens or sum(synth.prefill_lengths()))
    metric = "MoE-layer tokens/sec"

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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    li = synth.make_layer(shape, seed=0, tokens=args.tokens)
    if world > 1:  # each rank its own token batch (weak scaling)
        li.x = synth.gen_tokens(shape, args.tokens, seed=100 + rank, mu=li.mu)
        run_expert_parallel(args, shape, li, metric, rank, world, local, dist)
        return
    eng = L.Engine(local, max_layers=MAX_COPIES)
    eng.upload_layer(li)
    cfg = L.Engine.cfg(shape)
    T, H, K = args.tokens, shape.hidden, shape.top_k
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
        eng.upload_layer(li, layer=layer)
    cfgs = [cfg] + [L.Engine.cfg(shape, layer=layer) for layer in range(1, copies)]
    calls = [0]

    def next_cfg():
        calls[0] += 1
        return cfgs[(calls[0] - 1) % copies]

    def step():
        eng.forward(next_cfg(), x, T, y_bf16=y, ids=ids, w=w, stream=sp)

    for _ in range(args.warmup):
        step()
    eng.sync(sp)
    launches_per_step = eng.launches()

    # ---- device-timed region: inputs resident in HBM ----
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    eng.sync(sp)
    ms = start.elapsed_time(end)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = T * args.steps * world / (ms / 1000.0)

    # ---- per-stage breakdown: the same steps again with events between the
    # stages (kept out of the headline region above) ----
    eng.profile_enable(args.steps)
    for _ in range(args.steps):
        step()
    eng.sync(sp)
    stage_ms, prof_calls = eng.profile_read()
    eng.profile_enable(0)

    # ---- end to end through the host-buffer C-ABI call ----
    xh = torch.from_numpy(li.x.view(np.int16)).pin_memory()
    yh = torch.empty((T, H), dtype=torch.int16).pin_memory()
    idsh = torch.empty((T, K), dtype=torch.int32).pin_memory()
    wh = torch.empty((T, K), dtype=torch.float32).pin_memory()
    lib = L.load()
    import ctypes as C

    def step_host():
        ok = lib.moe_b200_layer_forward_host(eng.h, C.byref(next_cfg()), xh.data_ptr(), T, yh.data_ptr(), None,
                                             idsh.data_ptr(), wh.data_ptr(), None, eng.err)
        if not ok:
            raise L.MoEError(eng.err.value.decode())

    for _ in range(10):
        step_host()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e2e_steps = max(200, args.steps)  # host wall clock: a longer window for a steadier figure
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_host()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = T * e2e_steps * world / e2e_s

    # ---- roofline of the dominant kernel (gate/up grouped GEMM) ----
    counts = eng.read(L.BUF_GROUP_COUNT, (shape.experts,), np.uint32)
    distinct = int((counts > 0).sum())
    P = T * K
    # algorithmic bytes: MXFP4 weights of the experts routed to (17 bytes per
    # 32 elements) + the permuted activation rows in + the intermediate rows
    # out, both at 2 bytes per element (bf16, or the E4M3 hi/lo pair)
    Kp = H
    Ip = shape.intermediate
    gu_weight_bytes = distinct * 2 * shape.intermediate * H * 17 / 32
    gu_bytes = gu_weight_bytes + P * Kp * 2 + P * Ip * 2
    gu_ms = stage_ms["gate_up"] / max(prof_calls, 1)
    hbm, bf16, peak_kind = measured_peaks()
    achieved = gu_bytes / (gu_ms / 1000.0) / 1e9
    dn_ms = stage_ms["down"] / max(prof_calls, 1)
    dn_bytes = distinct * shape.intermediate * H * 17 / 32 + P * Ip * 2 + P * H * 4

    result = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": config_dict(shape, args, copies, touched),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2 + T * K * 8},
        "roofline": {"kernel": "gemm_bs_kernel<gate_up>", "bound": "hbm", "achieved": achieved, "peak": hbm,
                     "unit": "GB/s", "frac": achieved / hbm, "peak_source": peak_kind,
                     "traffic": profiled_traffic(args), "algorithmic_bytes_per_launch": gu_bytes,
                     "launch_ms": gu_ms, "distinct_experts": distinct},
        "stages_ms_per_step": {k: v / max(prof_calls, 1) for k, v in stage_ms.items()},
        "down_gemm": {"achieved_gbs": dn_bytes / (dn_ms / 1000.0) / 1e9, "launch_ms": dn_ms},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        li_cpu = synth.make_layer(shape, seed=0, tokens=args.tokens)
        result["cpu_baseline"] = cpu_baseline(li_cpu)
    if rank == 0:
        print(json.dumps(result), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
