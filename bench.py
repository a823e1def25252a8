"""Benchmark: batch-1 decode tok/s of the MiracleReasoning token loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config heavy] [--impl cuda|reference] [--replicas]

Headline workload: heavy-medium-2.0 (the largest
configuration one B200 holds: 36.5B parameters, 73 GB of BF16 weights),
random-init weights built in HBM by the seeded counter-hash generator, context
32768, a 4096-token prompt, then greedy decode.  A STEP is one decode token
(the whole model).  W untimed steps, then exactly K timed steps, bracketed by
a barrier and a device synchronize, timed with CUDA events on the engine's
stream (inside mr_model_bench_decode); the max over ranks is taken.  The
weights (20+ GB read per token) are far larger than L2, so every step streams
them from HBM.

Printed JSON line keys, beyond the driver contract's:
  roofline      algorithmic bytes per step (every weight read once + KV rows
                read and written) / measured step time, against
                MEASURED_PEAKS.json; traffic = DRAM bytes from a committed ncu
                summary when there is one (traffic_source names it)
  e2e           the same tok/s through the public Python API (model.decode:
                token id host->device, float32 logits device->host each step)
  prefill       prompt tok/s (batched tensor-core prefill for BF16 models of
                the grouped-query and latent families, else token by token)
  check         16 greedy ids and a logits checksum from a fixed 32-token
                prompt: the same on every N
  per_config    the same measurement for nano15, nano17, lite and lighting
                at their own BASELINE workloads
  cpu_baseline  the reference's CPU implementation on this host (its own
                kernels.cl compiled for the host, driven by the restated token
                loop with its LRU weight cache), on a bounded sample

N > 1: one process per GPU (torchrun).  By default the N GPUs decode ONE
sequence (tensor parallel: every projection and the lm_head split by output
row, attention by KV head, exchange words stored into every rank's memory over
NVLink; Heavy Medium: expert parallel, experts by id modulo the ranks; strong
scaling), value = that sequence's tokens / max time over ranks.  --replicas:
one independent sequence per GPU (weak scaling, no data-path collective).

--impl reference: the reference CPU implementation alone (rank 0 only), on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PACKAGE = "miraclereasoning-cpu_b200"
FALLBACK_HBM_GBS = 6650.0


def _pkg(name=""):
    return importlib.import_module(PACKAGE + ("." + name if name else ""))


# ---- distributed plumbing (replicas) ------------------------------------------------
class Ranks:
    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.dist = dist

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, value):
        if not self.dist:
            return value
        import torch
        t = torch.tensor([value], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_gather(self, data):
        items = [None] * self.world
        self.dist.all_gather_object(items, data)
        return items

    def close(self):
        if self.dist:
            self.dist.barrier()
            self.dist.destroy_process_group()


# ---- roofline bookkeeping ----------------------------------------------------------
def weight_bytes(config, stored="BF16", active_experts=None):
    """Bytes of every weight a decode step reads once (tied head = embed).

    Heavy Medium reads, per layer and inner loop, its attention and router
    matrices, the shared experts and the routed experts it chose:
    ``active_experts`` = the mean number chosen per (layer, loop)."""
    shapes = _pkg("weights").expected_shapes(config)
    total = 0
    expert = 0
    for name, shape in shapes.items():
        n = math.prod(shape) * (2 if (stored == "BF16" and len(shape) == 2) else 4)
        if ".experts." in name:
            if name.startswith("layers.0.experts.0."):
                expert += n
            continue
        if config.family == "heavy-medium-2.0" and name.startswith("layers."):
            n *= config.inner_loop_steps  # both inner loops read the layer's weights
        total += n
    if config.family == "heavy-medium-2.0":
        total += expert * active_experts * config.layers * config.inner_loop_steps
    # the embedding is read twice: one row for the input, the whole matrix for the tied head
    return total + config.hidden_size * (2 if stored == "BF16" else 4)


def kv_bytes(config, context, position):
    """float32 K/V bytes attended (read) and appended (written) at `position`."""
    total = 0
    if config.family == "heavy-medium-2.0":
        # per layer and inner loop: the local window's rows, every block mean (keys
        # and values), the newest block's rows for its mean, the appended row
        width = config.kv_heads * config.head_dim
        block = config.source["long_context"]["global_block_size"]
        rows = min(position + 1, config.window) + (position + block) // block + position % block + 1 + 1
        return config.layers * config.inner_loop_steps * rows * width * 2 * 4
    for layer in range(config.layers):
        width = config.layer_kv_heads(layer) * config.head_dim
        cap = min(config.layer_window(layer) or context, context)
        rows = min(position + 1, cap)
        total += rows * width * 2 * 4 + width * 2 * 4
    return total


def measured_hbm():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(config_name):
    """DRAM bytes per decode step from a committed ncu summary (profiles/), with the
    summary's name: a separate capture, not measured in this run."""
    for path in sorted((REPO / "profiles").glob(f"*_{config_name}.md")):
        for line in path.read_text().splitlines():
            if line.startswith(("traffic_bytes_per_launch:", "traffic_bytes_per_step:")):
                return float(line.split(":", 1)[1].strip()), f"profiles/{path.name} (ncu, separate capture)"
    return None, None


def launches_per_step(config, expert_parallel=False):
    """Kernels one decode step launches: the persistent decode kernel once, or
    Heavy Medium's device step (embedding row; per layer and inner loop 6
    kernels: q | latent, sparse attention, o, router + routing, gate | up,
    down + combine; expert parallel: gate | up, down, the flag kernel and the
    combine, so 8; then the head with its norm and the greedy argmax)."""
    if config.family == "heavy-medium-2.0":
        return 1 + (8 if expert_parallel else 6) * config.layers * config.inner_loop_steps + 2
    return 1


def mean_active_experts(model):
    """Heavy Medium: routed experts chosen per (layer, inner loop), averaged
    over the last decoded token's decisions (read back from the device)."""
    import ctypes as C
    c, s = model.config, model.config.source
    max_k = s["router_top_k_max"]
    experts, weights = (C.c_int * max_k)(), (C.c_float * max_k)()
    counts = []
    for layer in range(c.layers):
        for loop in range(c.inner_loop_steps):
            _pkg("_native").call("mr_model_last_experts", model._handle, layer, loop, experts, weights, max_k)
            counts.append(sum(1 for e in experts[:max_k] if e >= 0))
    return sum(counts) / len(counts)


# ---- clocks ------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device, self.proc, self.path = device, None, Path(f"/tmp/mr_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r.split(", ") for r in self.path.read_text().splitlines() if r.count(",") >= 8]
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ---- CPU baseline: the reference implementation on host cores -------------------------
def _reference_backend():
    from oracle.host_backend import HostBackend
    try:
        return HostBackend("reference"), "reference"
    except Exception:
        return HostBackend("oracle"), "port"


def cpu_reference_seconds(config, context, prompt, tokens, stored="BF16"):
    """Seconds per decode token of the reference CPU path: its own kernels.cl
    (oracle/_ref), driven by the restated token loop incl. the 256 MiB LRU
    weight cache, over the synthetic weights (all generated before the first
    token, so that no timed token pays for generating a weight: the reference
    would read them from its checkpoint's mmap)."""
    from oracle.reference_model import ReferenceModel
    backend, kind = _reference_backend()
    weights = _pkg("synthetic").synthetic_weights(config, stored)
    model = ReferenceModel(config, weights, backend=backend, context_length=context)
    logits = model.prefill(prompt)
    logits = model.decode(int(np.argmax(logits)))  # every weight this path reads is generated by now
    start = time.perf_counter()
    for _ in range(tokens):
        logits = model.decode(int(np.argmax(logits)))
    return (time.perf_counter() - start) / tokens, kind


def cpu_baseline(name, tokens):
    """The reference CPU path's decode tok/s on this host for configuration
    `name`, a bounded sample: `tokens` greedy tokens after a 4-token prompt;
    Heavy Medium (36.5B) on models of 1 and 2 layers of its shape, the token
    time taken as t1 + (layers - 1) * (t2 - t1)."""
    import dataclasses
    syn = _pkg("synthetic")
    config = syn.config_for(name)
    context = syn.WORKLOADS[name][0]
    stored = syn.STORED_DTYPE[name]
    prompt = list(syn.prompt_ids(config.vocab_size, 4))
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    t0 = time.perf_counter()
    if config.family == "heavy-medium-2.0":
        t1, kind = cpu_reference_seconds(dataclasses.replace(config, layers=1), 64, prompt, tokens, stored)
        t2, _ = cpu_reference_seconds(dataclasses.replace(config, layers=2), 64, prompt, tokens, stored)
        seconds = t1 + (config.layers - 1) * max(t2 - t1, 0.0)
        sample = (f"{tokens} greedy decode tokens after a 4-token prompt (+1 untimed) on models of 1 and 2 "
                  f"layers of the {name} shape; token time t1 + {config.layers - 1} * (t2 - t1) = {seconds:.2f} s")
    else:
        seconds, kind = cpu_reference_seconds(config, context, prompt, tokens, stored)
        sample = f"{tokens} greedy decode tokens after a 4-token prompt (+1 untimed) of the {name} model"
    return {"value": round(1.0 / seconds, 4), "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{sample} ({time.perf_counter() - t0:.1f} s of CPU work)"}


# ---- the CUDA measurement -------------------------------------------------------------
def build_model(name, ranks, mode):
    """The configuration's synthetic model: one per GPU (single / replicas) or one
    sequence over all ranks (split: tensor parallel, expert parallel for Heavy)."""
    syn = _pkg("synthetic")
    config = syn.config_for(name)
    context, prompt_len, _ = syn.WORKLOADS[name]
    backend = _pkg("backend").CUDABackend(device_index=ranks.local)
    kwargs = {"stored": syn.STORED_DTYPE[name], "backend": backend, "context_length": context}
    if mode == "split":
        kwargs["tensor_parallel"] = (ranks.rank, ranks.world, ranks.all_gather)
    seed = ranks.rank if mode == "replicas" else 0
    model = _pkg("model").MiracleModel.synthetic(config, seed=seed, **kwargs)
    prompt = syn.prompt_ids(config.vocab_size, prompt_len, seed=1 + (ranks.rank if mode == "replicas" else 0))
    return model, backend, config, context, prompt


def measure(name, args, ranks, mode, steps, warmup, sample_clocks):
    """One configuration: prefill tok/s, device-timed decode (W warm-up, K timed
    steps, CUDA events on the engine stream, max over ranks), the roofline,
    end-to-end decode through the Python API, and a determinism check (16
    greedy ids and a logits checksum from a fixed 32-token prompt)."""
    import ctypes as C
    native = _pkg("_native")
    model, backend, config, context, prompt = build_model(name, ranks, mode)
    stored = _pkg("synthetic").STORED_DTYPE[name]
    split = mode == "split"
    sequences = ranks.world if mode == "replicas" else 1
    heavy = config.family == "heavy-medium-2.0"
    if len(prompt) + 1 + warmup + steps > context:
        raise SystemExit("warmup + steps exceed the context window")

    # prefill: batched on the tensor cores for BF16 models of the engine families (timed
    # after one untimed pass: workspace allocation), else token by token (timed on its only pass)
    batched = C.c_int(0)
    native.call("mr_model_set_batched_prefill", model._handle, 1, C.byref(batched))
    serial = not batched.value
    if not serial:
        model.prefill(prompt)
        model.reset()
    backend.finish()
    ranks.barrier()
    t0 = time.perf_counter()
    logits = model.prefill(prompt)
    prefill_s = ranks.max(time.perf_counter() - t0)
    token = int(np.argmax(logits))

    # device-resident greedy decode: W warm-up steps, then exactly K timed steps
    ms = C.c_float()
    native.call("mr_model_bench_decode", model._handle, token, warmup, C.byref(ms))
    first_position = model.position
    clocks = ClockSampler(ranks.local) if sample_clocks else None
    if clocks:
        clocks.__enter__()
    ranks.barrier()
    backend.finish()
    native.call("mr_model_bench_decode", model._handle, token, steps, C.byref(ms))
    backend.finish()
    ranks.barrier()
    device_ms = ranks.max(ms.value)
    active = mean_active_experts(model) if heavy else None

    # end to end through the public API at the workload's positions (continuing after the
    # timed steps): token id in, float32 logits out, every step
    e2e_steps = min(steps, 128)
    logits = np.eye(1, config.vocab_size, token, dtype=np.float32)[0]
    ranks.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        logits = model.decode(int(np.argmax(logits)))
    e2e_s = ranks.max(time.perf_counter() - t0)
    e2e_first = model.position - e2e_steps
    if clocks:  # the same decode load for ~1.5 s more under the sampler (the same calls on every rank)
        step_ms = device_ms / steps
        extra = max(16, min(1024, context - 16, int(1.5e3 / step_ms)))
        for _ in range(max(1, math.ceil(1.5e3 / (step_ms * extra)))):
            model.reset()
            model.prefill(prompt[:8])
            native.call("mr_model_bench_decode", model._handle, token, extra, C.byref(ms))
        clocks.__exit__(None, None, None)

    # determinism check: identical on every N for the same configuration
    model.reset()
    logits = model.prefill(prompt[:32])
    ids = []
    for _ in range(16):
        ids.append(int(np.argmax(logits)))
        logits = model.decode(ids[-1])
    check = {"prompt": "first 32 ids of the workload prompt", "greedy_ids": ids,
             "logits_checksum": float(np.float64(logits.astype(np.float64).sum()))}

    # roofline: algorithmic bytes per step / device step time
    positions = range(first_position, first_position + steps)
    step_bytes = weight_bytes(config, stored, active) + sum(kv_bytes(config, context, p) for p in positions) / steps
    step_s = device_ms / 1e3 / steps
    peak, peak_kind = measured_hbm()
    per = "step"
    if split and heavy:  # attention replicated, experts split: the whole job's bytes against N peaks
        peak *= ranks.world
        per = f"job ({ranks.world} GPUs, peak x {ranks.world})"
    elif split:  # each GPU streams its slice of the weights and KV rows
        step_bytes /= ranks.world
        per = "GPU"
    achieved = step_bytes / step_s / 1e9
    traffic, traffic_source = ncu_traffic(name)
    parallelism = {"single": "single", "replicas": "replicas"}.get(
        mode, f"ep{ranks.world}" if heavy else f"tp{ranks.world}")
    result = {
        "value": round(sequences * steps / (device_ms / 1e3), 2), "unit": "tok/s",
        "ms_per_step": round(device_ms / steps, 5),
        "workload": f"{name}: {config.family} decode, {stored} weights "
                    f"({weight_bytes(config, stored, active) / 1e9:.3f} GB/step"
                    + (f" at {active:.2f} routed experts per layer and loop" if active else "")
                    + f"), greedy, positions {first_position}..{first_position + steps - 1}",
        "context": context, "prompt": len(prompt), "weights_dtype": stored, "parallelism": parallelism,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind, "bytes_per_step": int(step_bytes),
                     "per": per, "traffic": None if split else traffic,
                     "traffic_source": None if split or traffic is None else traffic_source},
        "e2e": {"value": round(sequences * e2e_steps / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * config.vocab_size, "steps": e2e_steps,
                "positions": f"{e2e_first}..{e2e_first + e2e_steps - 1}",
                "path": "MiracleModel.decode (Python API -> C ABI), logits to host each step"},
        "prefill": {"value": round(sequences * len(prompt) / prefill_s, 2), "unit": "tok/s", "tokens": len(prompt),
                    "note": ("batched prefill (heavy_prefill.cuh): tcgen05 GEMMs (BF16 weights x FP32 activations "
                             "split in three BF16 parts), routed experts as grouped GEMMs over the tokens sorted "
                             "by expert, sparse attention per token; logits of the last token to host"
                             if batched.value and heavy else
                             "batched prefill: tensor-core GEMMs (BF16 weights x FP32 activations split in three "
                             "BF16 parts) + causal attention over the chunk, logits of the last token to host"
                             if batched.value else
                             "prompt token by token through the device token step (heavy.cu kernels)"
                             if heavy else "prompt runs through the decode kernel token by token")},
        "check": check,
        "gpu_launches": steps * launches_per_step(config, split and heavy),
    }
    if clocks:
        result["clocks"] = clocks.summary()
    del model
    import gc
    gc.collect()
    return result


HEADLINE = "heavy"
PER_CONFIG = ("nano15", "nano17", "lite", "lighting")
PER_CONFIG_STEPS = {"nano15": 64, "nano17": 128, "lite": 128, "lighting": 96, "heavy": 32}


def profile_config(args):
    """The configuration of a profiling run: the benchmark's, or (--layers / --context)
    a reduced model of the same per-layer shape, so that an ncu capture holds a few GB."""
    import dataclasses
    syn = _pkg("synthetic")
    config = syn.config_for(args.config)
    context, prompt_len, _ = syn.WORKLOADS[args.config]
    if args.layers:
        config = dataclasses.replace(config, layers=args.layers,
                                     global_layers=tuple(g for g in config.global_layers if g <= args.layers))
    return config, (args.context or context), prompt_len


def run_profile_case(args):
    """The benchmark workload cut to a few decode steps, for ncu captures."""
    import ctypes as C
    syn = _pkg("synthetic")
    config, context, prompt_len = profile_config(args)
    prompt_len = args.profile_prompt or prompt_len
    backend = _pkg("backend").CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    model = _pkg("model").MiracleModel.synthetic(config, stored=syn.STORED_DTYPE[args.config], backend=backend,
                                                 context_length=context)
    logits = model.prefill(syn.prompt_ids(config.vocab_size, prompt_len, seed=1))
    ms = C.c_float()
    import torch  # the profiler range (ncu --profile-from-start off) covers the decode steps only
    backend.finish()
    torch.cuda.profiler.start()
    _pkg("_native").call("mr_model_bench_decode", model._handle, int(np.argmax(logits)), args.profile_steps,
                         C.byref(ms))
    torch.cuda.profiler.stop()
    print(json.dumps({"profile_case": args.config, "prompt": prompt_len, "decode_steps": args.profile_steps,
                      "position": model.position}))
    return 0


def run_profile_prefill(args):
    """Prefill of the benchmark prompt, repeated, for ncu captures of the
    batched prefill kernels; prints the wall time of each (not a bench value)."""
    syn = _pkg("synthetic")
    config, context, prompt_len = profile_config(args)
    prompt_len = args.profile_prompt or prompt_len
    backend = _pkg("backend").CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    model = _pkg("model").MiracleModel.synthetic(config, stored=syn.STORED_DTYPE[args.config], backend=backend,
                                                 context_length=context)
    prompt = syn.prompt_ids(config.vocab_size, prompt_len, seed=1)
    times = []
    import torch  # the profiler range (ncu --profile-from-start off) covers the last prefill only
    for i in range(args.profile_prefill):
        model.reset()
        backend.finish()
        last = i == args.profile_prefill - 1
        if last:
            torch.cuda.profiler.start()
        t0 = time.perf_counter()
        model.prefill(prompt)
        backend.finish()
        times.append(round((time.perf_counter() - t0) * 1e3, 3))
        if last:
            torch.cuda.profiler.stop()
    print(json.dumps({"profile_prefill": args.config, "prompt": prompt_len, "ms": times}))
    return 0


def run_trace(args, steps=8):
    """Per-phase timing of decode steps from the kernel's globaltimer stamps.

    Phases are not separated by grid barriers: every CTA starts a phase when it
    has finished the previous one and its input words carry the expected tag.
    Per phase kind (median over CTAs and steps, us): `input` = wait for the
    input words (plus the group's weight pieces) after the CTA finished the
    previous phase, `norm`, `compute`, `tail` (epilogue, record waits), and
    `critical` = how far the phase moves the slowest CTA's finish time.
    """
    import ctypes as C
    syn = _pkg("synthetic")
    native = _pkg("_native")
    config, context, prompt_len = profile_config(args)
    backend = _pkg("backend").CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    model = _pkg("model").MiracleModel.synthetic(config, stored=syn.STORED_DTYPE[args.config], backend=backend,
                                                 context_length=context)
    prompt_len = args.profile_prompt or prompt_len
    token = int(np.argmax(model.prefill(syn.prompt_ids(config.vocab_size, prompt_len, seed=1))))
    if config.family == "heavy-medium-2.0":
        return trace_heavy(args, model, token, steps)
    kinds = ["qkv", "attn", "o", "gate_up", "down"] * config.layers + ["head"]
    stamps_per_cta = 6
    capacity = 1 + len(kinds) * (200 * stamps_per_cta + 1)
    stamps = (C.c_uint64 * capacity)()
    phases, grid = C.c_int(), C.c_int()
    per_kind, totals = {}, []
    for _ in range(steps):
        native.call("mr_model_trace_decode", model._handle, token, stamps, capacity, C.byref(phases), C.byref(grid))
        g = grid.value
        rec = g * stamps_per_cta + 1
        t = np.frombuffer(stamps, dtype=np.uint64, count=1 + phases.value * rec).astype(np.int64)
        launch = t[0]
        prev_done = np.full(g, launch)
        prev_max = launch
        for k in range(phases.value):
            raw = t[1 + k * rec: 1 + (k + 1) * rec][:g * stamps_per_cta].reshape(g, stamps_per_cta)
            done = raw[:, 3]
            live = raw[:, 0] > 0  # CTAs that worked in this phase
            entry = per_kind.setdefault(kinds[k], {"input": [], "norm": [], "compute": [], "tail": [],
                                                   "critical": [], "piece_wait": [], "late_pieces": []})
            if live.any():
                r = raw[live]
                entry["input"].append(np.median(r[:, 0] - prev_done[live]))
                entry["norm"].append(np.median(r[:, 1] - r[:, 0]))
                entry["compute"].append(np.median(r[:, 2] - r[:, 1]))
                entry["tail"].append(np.median(r[:, 3] - r[:, 2]))
                entry["piece_wait"].append(np.median(r[:, 4]))
                entry["late_pieces"].append(1e3 * np.median(r[:, 5]))  # reported /1e3 below
            entry["critical"].append(done.max() - prev_max)
            prev_max = done.max()
            prev_done = done
        totals.append(prev_max - launch)
    report = {"config": args.config, "position": model.position, "steps": steps,
              "step_us": round(float(np.median(totals)) / 1e3, 2),
              "legend": "us, median over working CTAs: input = wait for the phase's input words after finishing the "
                        "previous phase; norm; compute (dot products / attention); tail (epilogue, record waits); "
                        "critical = advance of the slowest CTA's finish; piece_wait = thread 0 waiting for weight "
                        "pieces; late_pieces = pieces not yet in shared memory when first needed",
              "phases": {}}
    for kind, entry in per_kind.items():
        report["phases"][kind] = {k: round(float(np.median(v)) / 1e3, 3) if v else 0.0 for k, v in entry.items()}
        report["phases"][kind]["count_per_step"] = len(entry["critical"]) // steps
    print(json.dumps(report, indent=1))
    return 0


HEAVY_KERNELS = ["q|latent", "attention", "o", "router+route", "gate_up", "down+combine"]


def trace_heavy(args, model, token, steps):
    """Heavy Medium: the time each kernel of the token step adds to the
    critical path (completion stamp minus the previous kernel's), median over
    steps and (layer, inner loop), us; plus the step time with and without the
    stamp kernels (each stamp is one more tiny launch).  For every probed
    kernel, its probes relative to the previous kernel's completion: first CTA
    start, first CTA past the dependency wait, last CTA done staging its input,
    last CTA done with its main loop, last CTA exit (negative: before the
    previous kernel completed)."""
    import ctypes as C
    native = _pkg("_native")
    c = model.config
    loops = c.layers * c.inner_loop_steps
    kinds = ["embed"] + HEAVY_KERNELS * loops + ["head"]
    probed = len(HEAVY_KERNELS) * loops + 1
    nstamps = len(kinds) + 8
    capacity = nstamps + 8 * probed
    stamps = (C.c_uint64 * capacity)()
    phases, grid = C.c_int(), C.c_int()
    per_kind, probes, totals = {}, {}, []
    points = ["start", "waited", "staged", "main", "exit", "x5", "x6", "x7"]
    for _ in range(steps):
        native.call("mr_model_trace_decode", model._handle, token, stamps, capacity, C.byref(phases), C.byref(grid))
        t = np.frombuffer(stamps, dtype=np.uint64, count=capacity).astype(np.int64)
        if phases.value != len(kinds):
            raise SystemExit(f"trace: {phases.value} kernels, expected {len(kinds)}")
        for kind, dt in zip(kinds, np.diff(t[:phases.value + 1])):
            per_kind.setdefault(kind, []).append(dt)
        totals.append(t[phases.value] - t[0])
        pr = t[nstamps:].reshape(probed, 8)
        for i in range(probed):
            stamp_index = i + 2  # kernel kinds[i + 1] (the embedding row is not probed) completes at t[i + 2]
            prev = t[stamp_index - 1]
            kind = kinds[stamp_index - 1]
            rec = probes.setdefault(kind, {k: [] for k in points})
            for k, name in enumerate(points):
                if pr[i, k] not in (0, -1):
                    rec[name].append(pr[i, k] - prev)
    ms = C.c_float()
    native.call("mr_model_bench_decode", model._handle, token, steps, C.byref(ms))
    report = {"config": args.config, "position": model.position, "steps": steps,
              "step_us_traced": round(float(np.median(totals)) / 1e3, 1),
              "step_us_untraced": round(1e3 * ms.value / steps, 1),
              "legend": "us each kernel adds to the step (its completion stamp minus the previous one's), "
                        "median over steps and (layer, loop); total = per step; probes: us after the previous "
                        "kernel's completion (first CTA start / past the wait, last CTA staged / main loop done / exit)",
              "kernels": {k: {"median_us": round(float(np.median(v)) / 1e3, 2),
                              "total_us_per_step": round(float(np.sum(v)) / 1e3 / steps, 1),
                              **({"probes_us": {n: round(float(np.median(x)) / 1e3, 2) for n, x in probes[k].items()
                                                if x}} if k in probes else {})}
                          for k, v in per_kind.items()}}
    print(json.dumps(report, indent=1))
    return 0


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=32)
    parser.add_argument("--warmup", type=int, default=4)
    parser.add_argument("--config", default=HEADLINE, choices=["nano15", "nano17", "lite", "lighting", "heavy"],
                        help="the headline configuration (default: heavy-medium-2.0, the largest one a single "
                             "GPU holds)")
    parser.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    parser.add_argument("--cpu-tokens", type=int, default=3, help="decode tokens of each CPU baseline sample")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-per-config", action="store_true", help="measure the headline configuration only")
    parser.add_argument("--replicas", action="store_true",
                        help="with N > 1: N independent sequences, one per GPU (weak scaling); default: one "
                             "sequence over the N GPUs (tensor parallel; Heavy Medium: expert parallel)")
    parser.add_argument("--tp", action="store_true", help="accepted for compatibility: N > 1 splits by default")
    parser.add_argument("--trace", action="store_true",
                        help="print per-phase device timings of decode steps (phase tracing) and exit")
    parser.add_argument("--profile-steps", type=int, default=0,
                        help="profiling workload for ncu: build the model, prefill the prompt, run this many "
                             "decode steps, print no measurement")
    parser.add_argument("--profile-prompt", type=int, default=0,
                        help="with --profile-steps or --trace: a prompt of this many tokens instead of the "
                             "workload's")
    parser.add_argument("--layers", type=int, default=0,
                        help="profiling / tracing: a model of this many layers of the configuration's shape")
    parser.add_argument("--context", type=int, default=0, help="profiling / tracing: this context length")
    parser.add_argument("--profile-prefill", type=int, default=0,
                        help="profiling workload for ncu: build the model, prefill the prompt this many times")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    syn = _pkg("synthetic")
    config = syn.config_for(args.config)
    context, prompt_len, _ = syn.WORKLOADS[args.config]
    metric = f"batch-1 decode tok/s ({config.family}, context {context}, prompt {prompt_len})"

    if args.impl == "reference":
        # the reference's own CPU path on this host's cores (rank 0 only), a bounded sample
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        base = cpu_baseline(args.config, max(1, min(args.steps, args.cpu_tokens)))
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": base["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": max(1, min(args.steps, args.cpu_tokens)), "warmup": 1,
            "ms_per_step": round(1e3 / base["value"], 2), "higher_is_better": True,
            "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": f"{args.config} decode on host cores"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return 0

    if args.profile_steps:
        return run_profile_case(args)
    if args.profile_prefill:
        return run_profile_prefill(args)
    if args.trace:
        return run_trace(args)
    ranks = Ranks(args.gpus)
    mode = "single" if ranks.world == 1 else ("replicas" if args.replicas else "split")
    head = measure(args.config, args, ranks, mode, args.steps, args.warmup, sample_clocks=True)
    result = {
        "metric": metric, "value": head["value"], "unit": "tok/s", "n_gpus": ranks.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if mode == "split" else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": head["workload"], "context": head["context"], "prompt": head["prompt"],
                   "weights_dtype": head["weights_dtype"],
                   "l2": "inputs larger than L2 (weights stream from HBM every step)",
                   "parallelism": head["parallelism"]},
        "roofline": head["roofline"], "e2e": head["e2e"], "prefill": head["prefill"], "check": head["check"],
        "clocks": head.get("clocks"), "gpu_launches": head["gpu_launches"],
    }
    if not args.no_per_config:  # every other BASELINE configuration at its own workload
        per_config = {}
        for name in PER_CONFIG:
            if name == args.config:
                continue
            try:
                entry = measure(name, args, ranks, mode, PER_CONFIG_STEPS[name], args.warmup, sample_clocks=False)
            except Exception as exc:  # recorded, not hidden: the same on every rank
                entry = {"error": f"{type(exc).__name__}: {exc}"}
            if ranks.rank == 0 and not args.no_cpu_baseline and "error" not in entry:
                entry["cpu_baseline"] = cpu_baseline(name, args.cpu_tokens)
            per_config[name] = entry
        result["per_config"] = per_config
    if ranks.rank == 0 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.config, args.cpu_tokens)
    ranks.close()
    if ranks.rank == 0:
        print(json.dumps(result))
    return 0


if __name__ == "__main__":
    sys.exit(main())
