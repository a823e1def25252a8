"""Benchmark: batch-1 decode tok/s of the MiracleReasoning token loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config nano17] [--impl cuda|reference] [--tp]

Workload: flashnano-1.7, random-init BF16 weights
built in HBM by the seeded counter-hash generator, context 2048, a 512-token
prompt, then greedy decode.  A STEP is one decode token (the whole model, one
launch of the persistent decode kernel).  W untimed steps, then exactly K
timed steps, bracketed by a barrier and a device synchronize, timed with CUDA
events on the engine's stream (inside mr_model_bench_decode); the max over
ranks is taken.  The weights (0.5 GB) are larger than L2, so every step streams
them from HBM.

Printed JSON line keys, beyond the driver contract's:
  roofline      algorithmic bytes per step (every weight once + KV rows read
                and written) / measured step time, against MEASURED_PEAKS.json
  e2e           the same tok/s through the public Python API (model.decode:
                token id host->device, float32 logits device->host each step)
  prefill       prompt tok/s (batched tensor-core prefill for BF16 models, else token by token)
  cpu_baseline  the reference's CPU implementation on this host (its own
                kernels.cl compiled for the host, driven by the restated
                token loop with its LRU weight cache), on a bounded sample

N > 1: one process per GPU (torchrun), each rank decodes its own sequence on
its own GPU (independent replicas, weak scaling, no data-path collective);
value = tokens of all ranks / max time over ranks.  With --tp the N GPUs decode
ONE sequence together (tensor parallel: every projection and the lm_head split
by output row, attention by KV head, exchange words stored into every rank's
memory over NVLink; strong scaling), value = that sequence's tokens / max time.

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
    """DRAM bytes per launch of the decode kernel from the committed ncu summary, if any."""
    path = REPO / "profiles" / f"decode_step_kernel_{config_name}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip())
    return None


def launches_per_step(config, expert_parallel=False):
    """Kernels one decode step launches: the persistent decode kernel once, or
    Heavy Medium's device step (embedding row; per layer and inner loop 13
    kernels, 14 with the expert-parallel flag kernel; the head with its norm,
    greedy argmax)."""
    if config.family == "heavy-medium-2.0":
        return 1 + (14 if expert_parallel else 13) * config.layers * config.inner_loop_steps + 2
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
def cpu_reference_rate(config, context, prompt, tokens, stored="BF16"):
    """Decode tok/s of the reference CPU path: its own kernels.cl (oracle/_ref),
    driven by the restated token loop incl. the 256 MiB LRU weight cache."""
    from oracle.host_backend import HostBackend
    from oracle.reference_model import ReferenceModel
    try:
        backend, kind = HostBackend("reference"), "reference"
    except Exception:
        backend, kind = HostBackend("oracle"), "port"
    weights = _pkg("synthetic").synthetic_weights(config, stored)
    model = ReferenceModel(config, weights, backend=backend, context_length=context)
    logits = model.prefill(prompt)
    start = time.perf_counter()
    for _ in range(tokens):
        logits = model.decode(int(np.argmax(logits)))
    elapsed = time.perf_counter() - start
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return tokens / elapsed, kind, cores, elapsed


# ---- main --------------------------------------------------------------------------
def run_cuda(args, ranks):
    import ctypes as C
    syn = _pkg("synthetic")
    model_mod = _pkg("model")
    backend_mod = _pkg("backend")
    native = _pkg("_native")
    config = syn.config_for(args.config)
    context, prompt_len, decode_len = syn.WORKLOADS[args.config]
    stored = syn.STORED_DTYPE[args.config]
    if prompt_len + 1 + args.warmup + args.steps > context:
        raise SystemExit("warmup + steps exceed the context window")
    backend = backend_mod.CUDABackend(device_index=ranks.local)
    tp = args.tp and ranks.world > 1
    if tp:  # one model, one sequence, split over the ranks
        model = model_mod.MiracleModel.synthetic(config, stored=stored, seed=0, backend=backend,
                                                 context_length=context,
                                                 tensor_parallel=(ranks.rank, ranks.world, ranks.all_gather))
        prompt = syn.prompt_ids(config.vocab_size, prompt_len, seed=1)
    else:
        model = model_mod.MiracleModel.synthetic(config, stored=stored, seed=ranks.rank, backend=backend,
                                                 context_length=context)
        prompt = syn.prompt_ids(config.vocab_size, prompt_len, seed=1 + ranks.rank)
    sequences = 1 if tp else ranks.world

    # prefill, timed after one untimed pass (workspace allocation): batched on the
    # tensor cores for BF16 models of the grouped-query families; else token by
    # token (FlashLighting on the decode kernel, Heavy Medium on its device step),
    # which is timed on its only pass
    batched = C.c_int(0)
    if model._stepper is None and config.family != "heavy-medium-2.0":
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

    # device-resident decode: W warm-up steps, then exactly K timed steps
    ms = C.c_float()
    native.call("mr_model_bench_decode", model._handle, token, args.warmup, C.byref(ms))
    first_position = model.position
    with ClockSampler(ranks.local) as clocks:
        ranks.barrier()
        backend.finish()
        native.call("mr_model_bench_decode", model._handle, token, args.steps, C.byref(ms))
        backend.finish()
        ranks.barrier()
        device_ms = ranks.max(ms.value)
        active = mean_active_experts(model) if config.family == "heavy-medium-2.0" else None

        # end to end through the public API: token id in, float32 logits out, every step
        def end_to_end(logits):
            steps = min(args.steps, 128)
            ranks.barrier()
            t0 = time.perf_counter()
            for _ in range(steps):
                logits = model.decode(int(np.argmax(logits)))
            return steps, ranks.max(time.perf_counter() - t0)

        # a long token-by-token prompt: continue from here rather than run it again
        continue_e2e = serial and model.position + min(args.steps, 128) <= context
        if continue_e2e:
            e2e_steps, e2e_s = end_to_end(np.eye(1, config.vocab_size, token, dtype=np.float32)[0])
        # keep the same decode load under the clock sampler for ~1.5 s more (the same
        # number of calls on every rank: tensor-parallel ranks step together)
        step_ms = device_ms / args.steps
        extra_steps = max(16, min(1024, context - 16, int(1.5e3 / step_ms)))
        for _ in range(max(1, math.ceil(1.5e3 / (step_ms * extra_steps)))):
            model.reset()
            model.prefill(prompt[:8])
            native.call("mr_model_bench_decode", model._handle, token, extra_steps, C.byref(ms))
    clock_summary = clocks.summary()

    if not continue_e2e:
        model.reset()
        e2e_steps, e2e_s = end_to_end(model.prefill(prompt))

    # roofline
    positions = range(first_position, first_position + args.steps)
    step_bytes = weight_bytes(config, stored, active) + sum(kv_bytes(config, context, p) for p in positions) / args.steps
    step_s = device_ms / 1e3 / args.steps
    peak, peak_kind = measured_hbm()
    per = "step"
    if tp and config.family == "heavy-medium-2.0":  # attention replicated, experts split: the whole job's bytes
        peak *= ranks.world
        per = f"job ({ranks.world} GPUs, peak x {ranks.world})"
    elif tp:  # each GPU streams its slice of the weights and KV rows
        step_bytes /= ranks.world
        per = "GPU"
    achieved = step_bytes / step_s / 1e9
    value = sequences * args.steps / (device_ms / 1e3)
    result = {
        "metric": f"batch-1 decode tok/s ({config.family}, context {context}, prompt {prompt_len})",
        "value": round(value, 2), "unit": "tok/s", "n_gpus": ranks.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(device_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config}: {config.family} decode, {stored} weights "
                               f"({weight_bytes(config, stored, active) / 1e9:.3f} GB/step"
                               + (f" at {active:.2f} routed experts per layer and loop" if active else "")
                               + "), greedy, positions "
                               f"{first_position}..{first_position + args.steps - 1}",
                   "context": context, "prompt": prompt_len, "weights_dtype": stored,
                   "l2": "inputs larger than L2 (weights stream from HBM every step)",
                   "parallelism": (f"ep{ranks.world}" if config.family == "heavy-medium-2.0" else f"tp{ranks.world}")
                                  if tp else ("replicas" if ranks.world > 1 else "single")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "bytes_per_step": int(step_bytes), "per": per,
                     "traffic": None if tp else ncu_traffic(args.config)},
        "e2e": {"value": round(sequences * e2e_steps / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * config.vocab_size, "steps": e2e_steps,
                "path": "MiracleModel.decode (Python API -> C ABI), logits to host each step"},
        "prefill": {"value": round(sequences * prompt_len / prefill_s, 2), "unit": "tok/s",
                    "tokens": prompt_len,
                    "note": ("batched prefill: tensor-core GEMMs (BF16 weights x FP32 activations split in three BF16 "
                             "parts) + causal attention over the chunk, logits of the last token to host"
                             if batched.value else
                             "prompt token by token through the device token step (heavy.cu kernels)"
                             if config.family == "heavy-medium-2.0" else
                             "prompt runs through the decode kernel token by token")},
        "clocks": clock_summary,
        "gpu_launches": args.steps * launches_per_step(config, tp),
    }
    return result, config, context, prompt


def run_profile_case(args):
    """The benchmark workload cut to a few decode steps, for ncu captures."""
    import ctypes as C
    syn = _pkg("synthetic")
    config = syn.config_for(args.config)
    context, prompt_len, _ = syn.WORKLOADS[args.config]
    prompt_len = args.profile_prompt or prompt_len
    backend = _pkg("backend").CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    model = _pkg("model").MiracleModel.synthetic(config, stored=syn.STORED_DTYPE[args.config], backend=backend,
                                                 context_length=context)
    logits = model.prefill(syn.prompt_ids(config.vocab_size, prompt_len, seed=1))
    ms = C.c_float()
    _pkg("_native").call("mr_model_bench_decode", model._handle, int(np.argmax(logits)), args.profile_steps,
                         C.byref(ms))
    print(json.dumps({"profile_case": args.config, "prompt": prompt_len, "decode_steps": args.profile_steps,
                      "position": model.position}))
    return 0


def run_profile_prefill(args):
    """Prefill of the benchmark prompt, repeated, for ncu captures of the
    batched prefill kernels; prints the wall time of each (not a bench value)."""
    syn = _pkg("synthetic")
    config = syn.config_for(args.config)
    context, prompt_len, _ = syn.WORKLOADS[args.config]
    backend = _pkg("backend").CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    model = _pkg("model").MiracleModel.synthetic(config, stored=syn.STORED_DTYPE[args.config], backend=backend,
                                                 context_length=context)
    prompt = syn.prompt_ids(config.vocab_size, prompt_len, seed=1)
    times = []
    for _ in range(args.profile_prefill):
        model.reset()
        backend.finish()
        t0 = time.perf_counter()
        model.prefill(prompt)
        backend.finish()
        times.append(round((time.perf_counter() - t0) * 1e3, 3))
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
    config = syn.config_for(args.config)
    context, prompt_len, _ = syn.WORKLOADS[args.config]
    backend = _pkg("backend").CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    model = _pkg("model").MiracleModel.synthetic(config, stored=syn.STORED_DTYPE[args.config], backend=backend,
                                                 context_length=context)
    token = int(np.argmax(model.prefill(syn.prompt_ids(config.vocab_size, prompt_len, seed=1))))
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


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=480)
    parser.add_argument("--warmup", type=int, default=16)
    parser.add_argument("--config", default="nano17", choices=["nano15", "nano17", "lite", "lighting", "heavy"])
    parser.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    parser.add_argument("--cpu-tokens", type=int, default=12, help="decode tokens of the CPU baseline sample")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--tp", action="store_true",
                        help="with N > 1: the N GPUs decode one sequence, tensor-parallel (Heavy Medium: "
                             "expert-parallel); default: N replicas")
    parser.add_argument("--trace", action="store_true",
                        help="print per-phase device timings of decode steps (phase tracing) and exit")
    parser.add_argument("--profile-steps", type=int, default=0,
                        help="profiling workload for ncu: build the model, prefill the prompt, run this many "
                             "decode steps, print no measurement")
    parser.add_argument("--profile-prompt", type=int, default=0,
                        help="with --profile-steps: a prompt of this many tokens instead of the workload's")
    parser.add_argument("--profile-prefill", type=int, default=0,
                        help="profiling workload for ncu: build the model, prefill the prompt this many times")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    syn = _pkg("synthetic")

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        config = syn.config_for(args.config)
        context, prompt_len, _ = syn.WORKLOADS[args.config]
        steps = min(args.steps, args.cpu_tokens)
        prompt = syn.prompt_ids(config.vocab_size, 4)
        rate, kind, cores, elapsed = cpu_reference_rate(config, context, prompt, steps, syn.STORED_DTYPE[args.config])
        sample = (f"{steps} greedy decode tokens after a 4-token prompt (positions 4..{3 + steps}) of the "
                  f"{args.config} model; bounded sample of the {prompt_len}-token-prompt workload")
        print(json.dumps({
            "impl": "reference", "metric": f"batch-1 decode tok/s ({config.family}, context {context}, "
                                           f"prompt {prompt_len})",
            "value": round(rate, 4), "unit": "tok/s", "n_gpus": args.gpus, "steps": steps, "warmup": 0,
            "ms_per_step": round(1e3 * elapsed / steps, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.config} decode on host cores"},
            "cpu_baseline": {"value": round(rate, 4), "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": round(rate, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return 0

    if args.profile_steps:
        return run_profile_case(args)
    if args.profile_prefill:
        return run_profile_prefill(args)
    if args.trace:
        return run_trace(args)
    ranks = Ranks(args.gpus)
    result, config, context, prompt = run_cuda(args, ranks)
    if ranks.rank == 0 and not args.no_cpu_baseline:
        rate, kind, cores, elapsed = cpu_reference_rate(config, context, list(prompt[:4]), args.cpu_tokens,
                                                        syn.STORED_DTYPE[args.config])
        result["cpu_baseline"] = {
            "value": round(rate, 4), "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{args.cpu_tokens} greedy decode tokens after a 4-token prompt on the same model "
                      f"({elapsed:.1f} s of CPU work)"}
    ranks.close()
    if ranks.rank == 0:
        print(json.dumps(result))
    return 0


if __name__ == "__main__":
    sys.exit(main())
