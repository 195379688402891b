#!/usr/bin/env python3
"""RVQ decode benchmark (B200, sm_100a).

Workload (one GPU): the ping-pong slot fill of a Qwen-style decoder block --
hidden 2560, intermediate 9728, 32 query / 8 KV heads of 128 -- whose 7
projections are RVQ-compressed (K=4 stages, 256 codes, d=8, per-row fp16
scales) and whose 4 norm weights are bf16 copies.  One step decodes one
layer into a bf16 slot: 100,925,440 weights, 252,375,040 algorithmic bytes
(slot writes + index reads + scale reads).  Steps cycle through 8 distinct
layers and 2 slots, so consecutive steps never find their inputs in L2
(every step touches > 250 MB against a 126 MB L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun, one process per GPU): every rank decodes its own layers
(weak scaling, no collective on the data path); the timed region is
bracketed by barriers and the slowest rank's time is reported.

Rank 0 prints one JSON line.  ``value`` is whole-job GB/s with inputs
resident in HBM; ``e2e`` is the same metric through the reference-facing
``decode_into`` API with the layer's compressed tensors copied from pinned
host memory and the decoded slot copied back every step; ``cpu_baseline``
times the CPU port of the reference's reconstruction on this host's cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "RVQ decode GB/s (% HBM peak); batch-1 ms/token at 1/2/4/8 B200"
WORKLOAD = ("config1 ping-pong slot fill: Qwen-style block hidden 2560 / intermediate 9728 / "
            "32q 8kv head 128, 7 RVQ projections (K=4, 256 codes, d=8, per-row fp16 scales) "
            "+ 4 bf16 norms -> bf16 slot")
N_LAYERS_ROTATED = 8
DECODE_KERNEL = "rvq_slot_kernel"           # what a layer plan launches (quad codes, fp16 codebook, bf16 slot)
# slot writes + code reads + scale reads of the 7 projections, plus the 4 bf16 norm copies
BYTES_PER_STEP = 252396544
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline sample budget (rank 0, N=1)")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch1", action="store_true",
                    help="skip the batch-1 generation ms/token leg")
    ap.add_argument("--no-overlap", action="store_true",
                    help="skip the config-1 ping-pong overlap leg")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        data = json.load(f)
    rec = data.get(kernel)
    return None if rec is None else rec.get("bytes_per_launch")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.path = None
        try:
            self.uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.uuid = None

    def start(self):
        if self.uuid is None:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", self.uuid, "-lms", "100", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        sm.append(float(parts[1]))
                        smax = float(parts[2])
                    except ValueError:
                        continue
                    for name, val in zip(names, parts[5:9]):
                        if val.lower().startswith("active"):
                            reasons.add(name)
            os.unlink(self.path)
        except OSError:
            return None
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    return world, rank, local


# ---------------------------------------------------------------------------
# CPU reference arm / baseline (the oracle's C port of the reference path)
# ---------------------------------------------------------------------------

def cpu_block_sample(frac_rows: float, seed: int = 0):
    """Entries of one config-1 block, each cut to its first `frac_rows` of
    output rows (a contiguous vector range of every index plane)."""
    from oracle.rvq_oracle import RVQEntryNP
    from rvq_b200 import synthetic
    art = synthetic.make_block_artifact(seed=seed)
    out = []
    for key, e in art["entries"].items():
        if e["method"] != "rvq_groupwise":
            continue
        rows, cols = e["shape"]
        keep_rows = max(1, int(rows * frac_rows))
        nvec = keep_rows * cols // 8
        cb = art["shared_codebooks"][e["codebook_id"]].float().numpy()
        idx = e["indices"][:, :nvec].contiguous().numpy()
        gv = int(e["group_size"]) // 8
        sc = e["scales"][: (nvec + gv - 1) // gv].float().numpy()
        ent = RVQEntryNP(indices=idx, codebook=cb, scales=sc, tail=sc[:0], d=8,
                         group_size=int(e["group_size"]), trimmed_numel=nvec * 8,
                         numel=nvec * 8)
        algo = nvec * 8 * 2 + idx.size + sc.size * 2
        out.append((ent, algo))
    return out


def time_cpu_port(sample, seconds: float, min_reps: int = 1):
    import numpy as np

    from oracle.c_oracle import decode_rvq_bits_c, max_threads
    from oracle.rvq_oracle import OUT_BF16
    threads = max_threads()
    bufs = [np.empty(e.numel, np.uint16) for e, _ in sample]
    algo = sum(a for _, a in sample)
    for (e, _), b in zip(sample, bufs):        # warm-up (page-in)
        decode_rvq_bits_c(e, OUT_BF16, nthreads=threads, out=b)
    reps, t0 = 0, time.perf_counter()
    while True:
        for (e, _), b in zip(sample, bufs):
            decode_rvq_bits_c(e, OUT_BF16, nthreads=threads, out=b)
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= seconds:
            break
    return algo * reps / el / 1e9, threads, reps, el, algo


def torch_block_sample(seed: int = 0):
    """The RVQ entries of one config-1 block as CPU torch tensors, with their
    codebooks and bf16 outputs, for the PyTorch restatement of the reference's
    ``_decode_rvq_into``."""
    from rvq_b200 import synthetic
    art = synthetic.make_block_artifact(seed=seed)
    items = []
    for key, e in art["entries"].items():
        if e["method"] != "rvq_groupwise":
            continue
        cb = art["shared_codebooks"][e["codebook_id"]].float()
        out = torch.empty(tuple(e["shape"]), dtype=torch.bfloat16)
        items.append((e, cb, out))
    return items


def time_torch_port(seconds: float, min_reps: int = 1):
    """The reference's PyTorch CPU reconstruction (oracle.torch_port restates
    infer_compressed_layerwise_single_slot.py:123-149) over whole config-1
    blocks, with every host thread; returns (GB/s, threads, blocks, s)."""
    from oracle.torch_port import decode_rvq_into
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    items = torch_block_sample()
    algo = sum(e["indices"].numel() + e["scales"].numel() * 2 + out.numel() * 2 for e, _, out in items)
    for e, cb, out in items:                 # warm-up (page-in, allocator)
        decode_rvq_into(e, cb, out)
    reps, t0 = 0, time.perf_counter()
    while True:
        for e, cb, out in items:
            decode_rvq_into(e, cb, out)
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= seconds:
            break
    return algo * reps / el / 1e9, threads, reps, el


def cpu_baselines(seconds: float):
    """Both CPU figures on this host: the C/OpenMP port (the stronger one,
    reported as ``value``) and the PyTorch restatement of the reference's own
    function (``torch_port``), each over whole config-1 blocks."""
    sample = cpu_block_sample(1.0)
    v, threads, reps, el, algo = time_cpu_port(sample, seconds)
    tv, tthreads, treps, tel = time_torch_port(seconds)
    return {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} full config-1 block decode(s) ({algo} algorithmic bytes each), "
                      f"C/OpenMP port of the reference reconstruction, bf16 out, {el:.1f} s",
            "torch_port": {"value": round(tv, 4), "unit": "GB/s", "cores": tthreads,
                           "sample": f"{treps} full config-1 block decode(s), PyTorch restatement of the "
                                     f"reference's _decode_rvq_into (same ops, torch.set_num_threads"
                                     f"({tthreads})), bf16 out, {tel:.1f} s"}}


def run_reference_arm(args, world, rank):
    """The reference's CPU reconstruction of the same workload as the GPU arm:
    every step decodes one whole config-1 block (7 projections) into bf16 on
    the host's cores with the C/OpenMP port; rank 0 only."""
    if rank != 0:
        return
    sample = cpu_block_sample(1.0)
    from oracle.c_oracle import decode_rvq_bits_c, max_threads
    from oracle.rvq_oracle import OUT_BF16
    import numpy as np
    threads = max_threads()
    bufs = [np.empty(e.numel, np.uint16) for e, _ in sample]
    algo = sum(a for _, a in sample)

    def step():
        for (e, _), b in zip(sample, bufs):
            decode_rvq_bits_c(e, OUT_BF16, nthreads=threads, out=b)

    for _ in range(max(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gbs = algo * args.steps / el / 1e9
    desc = (f"one whole config-1 block per step ({algo} algorithmic bytes: 7 projections, bf16 out), "
            f"C/OpenMP port of the reference reconstruction on {threads} host threads")
    tv, tthreads, treps, tel = time_torch_port(min(args.cpu_seconds, 10.0))
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": gpu_config(world),
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": desc,
                         "torch_port": {"value": round(tv, 4), "unit": "GB/s", "cores": tthreads,
                                        "sample": f"{treps} whole block(s) in {tel:.1f} s, PyTorch "
                                                  f"restatement of the reference's _decode_rvq_into"}},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def gpu_config(world: int) -> dict:
    """The workload description both arms print."""
    return {"workload": WORKLOAD, "bytes_per_step_per_gpu": BYTES_PER_STEP,
            "weights_per_step_per_gpu": 100925440, "layers_rotated": N_LAYERS_ROTATED,
            "slots": 2, "l2": "inputs larger than L2: >250 MB touched per step, 8 distinct layers rotated",
            "timed_region": "K steps replayed from one CUDA graph on the launching stream",
            "parallelism": f"independent per-GPU decode x{world}"}


def build_layers(device, n_layers):
    """n_layers distinct copies of one seeded block resident on the device,
    2 bf16 slots, and one LayerDecodePlan per layer (layer l -> slot l % 2)."""
    from rvq_b200 import synthetic
    from rvq_b200.engine import LayerDecodePlan
    art = synthetic.make_block_artifact(seed=0)
    cbs = {k: v.to(device, torch.float32) for k, v in art["shared_codebooks"].items()}
    rel = {}
    for key, e in art["entries"].items():
        rel[key.split("layers.0.")[-1]] = e
    slots = [{k: torch.empty(tuple(e["shape"]), dtype=torch.bfloat16, device=device)
              for k, e in rel.items()} for _ in range(2)]
    layers, plans = [], []
    for l in range(n_layers):
        dev_entries = {k: {ek: (ev.to(device) if torch.is_tensor(ev) else ev) for ek, ev in e.items()}
                       for k, e in rel.items()}
        layers.append(dev_entries)
        plans.append(LayerDecodePlan(list(dev_entries.items()), cbs, slots[l % 2]))
    return art, rel, cbs, slots, layers, plans


def time_device(plans, steps, warmup, stream, world):
    """W eager warm-up steps, then exactly K steps replayed from one CUDA graph
    (the same launches, without host launch gaps between them).  The graph is
    replayed once untimed first, so its upload and first-launch costs stay
    outside the timed region."""
    for s in range(warmup):
        plans[s % len(plans)].launch(stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for s in range(steps):
            plans[s % len(plans)].launch(stream.cuda_stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    with torch.cuda.stream(stream):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    del graph
    ms = start.elapsed_time(end)
    if world > 1:
        torch.distributed.barrier()
    return ms


def time_e2e(rel, cbs_host, device, steps, warmup, stream):
    """Reference-facing API end to end: every step uploads the layer's
    compressed tensors and codebooks from pinned host memory
    (infer_compressed_layerwise_triton.py:424-432), decodes them with
    decode_into per key (lines 161-176) and copies the decoded slot back to
    pinned host memory.  Steps are pipelined over three streams (upload,
    decode, download) with two buffer sets, so one step's upload and the
    previous step's download run while a decode runs (PCIe is full duplex);
    events order every reuse of a buffer set.  Timed from the first upload to
    the last download."""
    from rvq_b200.engine import decode_into
    host = {k: {ek: (ev.pin_memory() if torch.is_tensor(ev) else ev) for ek, ev in e.items()}
            for k, e in rel.items()}
    host_cbs = {k: v.float().pin_memory() for k, v in cbs_host.items()}
    sets = []
    for _ in range(2):
        dev = {k: {ek: (torch.empty_like(ev, device=device) if torch.is_tensor(ev) else ev)
                   for ek, ev in e.items()} for k, e in rel.items()}
        dev_cbs = {k: torch.empty_like(v, device=device) for k, v in host_cbs.items()}
        slot = {k: torch.empty(tuple(e["shape"]), dtype=torch.bfloat16, device=device) for k, e in rel.items()}
        back = {k: torch.empty(tuple(e["shape"]), dtype=torch.bfloat16).pin_memory() for k, e in rel.items()}
        ev = {n: torch.cuda.Event() for n in ("in", "cmp", "out")}
        sets.append({"dev": dev, "cbs": dev_cbs, "slot": slot, "back": back, "ev": ev, "used": False})
    h2d = sum(v.numel() * v.element_size() for e in host.values() for v in e.values() if torch.is_tensor(v))
    h2d += sum(v.numel() * v.element_size() for v in host_cbs.values())
    d2h = sum(v.numel() * v.element_size() for v in sets[0]["back"].values())
    launches = sum(1 for e in rel.values() if e["method"] != "bf16_raw")
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    s_cmp = stream

    def step(i):
        b = sets[i % 2]
        ev = b["ev"]
        if b["used"]:
            s_in.wait_event(ev["cmp"])              # the decode of step i - 2 has read these inputs
            s_cmp.wait_event(ev["out"])             # the download of step i - 2 has read this slot
        b["used"] = True
        with torch.cuda.stream(s_in):
            for k, v in host_cbs.items():
                b["cbs"][k].copy_(v, non_blocking=True)
            for k, e in host.items():
                for ek, hv in e.items():
                    if torch.is_tensor(hv):
                        b["dev"][k][ek].copy_(hv, non_blocking=True)
            ev["in"].record(s_in)
        s_cmp.wait_event(ev["in"])
        with torch.cuda.stream(s_cmp):
            for k, e in b["dev"].items():
                decode_into(e, b["cbs"], b["slot"][k])
            ev["cmp"].record(s_cmp)
        s_out.wait_event(ev["cmp"])
        with torch.cuda.stream(s_out):
            for k in b["slot"]:
                b["back"][k].copy_(b["slot"][k], non_blocking=True)
            ev["out"].record(s_out)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for i in range(steps):
        step(warmup + i)
    end.record(s_out)
    torch.cuda.synchronize()
    return start.elapsed_time(end), h2d, d2h, launches * steps


def overlap_leg(device):
    """Config 1's ping-pong overlap: the next layer decoded into the other slot
    on a low-priority side stream while the batch-1 bf16 block forward runs on
    the main stream, overlap = (t_dec + t_fwd - t_both) / min(t_dec, t_fwd).
    Reported with the decode on every SM (fastest alone) and with a CTA budget
    of half the SMs (the other half free for the forward's kernels)."""
    from rvq_b200 import bench_overlap
    try:
        half = torch.cuda.get_device_properties(device).multi_processor_count // 2
        res = {"all_sms": bench_overlap.run(30, device, max_ctas=0),
               "half_sms": bench_overlap.run(30, device, max_ctas=half)}
        for r in res.values():
            r.pop("workload", None)
            r.pop("timing", None)
        best = max(res, key=lambda k: res[k]["overlap"])
        return {"overlap": res[best]["overlap"], "config": best, **res,
                "definition": "(t_dec + t_fwd - t_both) / min(t_dec, t_fwd), us per layer, CUDA graphs on two "
                              "streams (forward high priority), config-1 block, bf16 forward on resident weights"}
    except Exception as exc:                     # reported in the line; the decode figures stand
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


def batch1_leg(world, device, peak):
    """Batch-1 greedy generation, ms/token (the metric's second half).  N=1:
    the 36-layer 2560/9728 model in every weight mode (dense bf16, slot
    decode + cuBLAS, fused table GEMV, fused exact-weight GEMV, fused table
    GEMV with the whole step as one persistent cooperative launch), each mode's
    ids checked against the drop-in engine (HF decoder layers on decoded
    slots, bit-identical to the oracle engine pinned to the reference
    engine's output), and the 64-layer 5120/25600 model; N>1: the 64-layer
    model tensor-parallel over the N GPUs (row-parallel outputs summed by peer
    stores over NVLink into every rank's landing buffer, rvq_b200/tp.py)."""
    from rvq_b200 import bench_generate, bench_tp
    out = {"prompt_tokens": 128, "new_tokens": 128, "timing": "device time per token, max over ranks",
           "tp_reduce": "push (peer stores into landing buffers)" if world > 1 else None,
           "data": "synthetic random-init weights generated on the GPU, seeded"}
    try:
        group = torch.distributed.group.WORLD if world > 1 else None
        if world == 1:
            out["config2_36_layers"] = bench_generate.run(36, 128, 128, 151936, reps=2, device=device,
                                                          hbm_gbs=peak)
        c4 = {}
        for mode in ("fused", "fused_exact") + (("fused_persistent",) if world == 1 else ()):
            c4[mode] = bench_tp.measure(bench_tp.SHAPE, 64, 151936, mode, device, group)
            c4[mode]["per_gpu_weight_GB/s"] = round(bench_tp.bytes_per_token(bench_tp.SHAPE, 64, 151936, world)
                                                    / (c4[mode]["ms_per_token"] * 1e6), 1)
            c4[mode]["roofline_frac"] = round(c4[mode]["per_gpu_weight_GB/s"] / peak, 4)
        out[f"config4_64_layers_tp{world}"] = c4
    except Exception as exc:                     # reported in the line; the decode figures above stand
        out["error"] = f"{type(exc).__name__}: {exc}"[:300]
    return out


def run_ours(args, world, rank, local):
    from rvq_b200 import _native
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    _native.load()
    if not _native.available():
        raise RuntimeError("rvq_b200 CUDA library has no usable sm_100 device")
    art, rel, cbs, slots, layers, plans = build_layers(device, N_LAYERS_ROTATED)
    bytes_per_step = plans[0].algorithmic_bytes
    if bytes_per_step != BYTES_PER_STEP:
        raise RuntimeError(f"block bytes {bytes_per_step} differ from the workload's {BYTES_PER_STEP}")
    launches_per_step = plans[0].launches
    stream = torch.cuda.Stream(device)

    sampler = ClockSampler(device) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ms = time_device(plans, args.steps, max(args.warmup, 3), stream, world)
    clocks = sampler.stop() if sampler else None

    ms_t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    total_bytes = bytes_per_step * args.steps * world
    gbs = total_bytes / (ms_max / 1e3) / 1e9
    per_launch_s = (ms / 1e3) / (args.steps * launches_per_step)
    achieved = bytes_per_step / launches_per_step / per_launch_s / 1e9
    peak, peak_kind = measured_peaks()

    e2e = None
    if rank == 0 or world > 1:
        e2e_ms, h2d, d2h, e2e_launches = time_e2e(rel, art["shared_codebooks"], device,
                                                  args.e2e_steps, 2, stream)
        e2e_t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        if world > 1:
            torch.distributed.all_reduce(e2e_t, op=torch.distributed.ReduceOp.MAX)
        e2e_gbs = bytes_per_step * args.e2e_steps * world / (float(e2e_t.item()) / 1e3) / 1e9
        e2e = {"value": round(e2e_gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
               "api": "rvq_b200.engine.decode_into per entry (reference-facing)",
               "pipelining": "upload, decode and download on three streams, two buffer sets",
               "gpu_launches": e2e_launches}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baselines(args.cpu_seconds)

    overlap = None
    if rank == 0 and world == 1 and not args.no_overlap:
        overlap = overlap_leg(device)

    batch1 = None
    if not args.no_batch1:
        batch1 = batch1_leg(world, device, peak)

    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms_max / args.steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": gpu_config(world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": profile_traffic(DECODE_KERNEL),
                     "kernel": DECODE_KERNEL,
                     "algorithmic_bytes_per_launch": bytes_per_step // launches_per_step},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clocks,
        "overlap": overlap,
        "batch1": batch1,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world, rank, local = dist_init(args)
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
