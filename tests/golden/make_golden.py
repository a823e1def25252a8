"""Generate the golden fixtures by running the REFERENCE implementation itself.

Run in a container that has the read-only reference checkout:

    python tests/golden/make_golden.py --reference-root DIR   (or MIRACLE_REFERENCE_ROOT=DIR)

The reference package (miracle_reasoning: model.py, config.py, weights.py) is
imported unmodified and driven with ``oracle.host_backend.HostBackend
("reference")``, i.e. the reference's own kernels.cl compiled for the host by
oracle/build.py.  Nothing of the reference is copied; only its outputs are
saved:

* ``kernels.npz`` — the kernel known-answer cases of tests/test_opencl.py:19-63
  (same seeds and shapes);
* ``configs.npz`` — RoPE inverse-frequency tables, native-name tables and
  expected shapes for every case configuration and several RoPE variants;
* ``micro_<case>.npz`` — per micro case (tests/golden/cases.py): all-token
  logits, chunked-prefill logits, cache state, discrete decisions (heavy
  top-k blocks, MoE experts and weights, latent positions), greedy and sampled
  ``generate`` ids;
* ``bench_<case>.npz`` — every benchmark architecture at full size with a
  short token window: leading logits, every 16th logit, top-64 ids/values,
  the greedy ids (Heavy Medium: also experts and kept blocks per layer/loop);
* ``prefill_<case>.npz`` — micro architectures with BF16 matrices and a
  48-token prompt: all-token logits, two-chunk logits, cache state, greedy
  decode steps after the prompt.

Discrete decisions are observed by wrapping the reference model's methods on
the instance (no reference source is changed).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from collections.abc import Mapping
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))
import cases  # noqa: E402
from oracle.host_backend import HostBackend  # noqa: E402


class RecordingWeights(Mapping):
    def __init__(self, inner, log):
        self.inner, self.log = inner, log

    def __iter__(self):
        return iter(self.inner)

    def __len__(self):
        return len(self.inner)

    def __contains__(self, key):
        return key in self.inner

    def __getitem__(self, key):
        self.log.append(key)
        return self.inner[key]


def _ref_modules(root):
    sys.path.insert(0, str(root))
    import miracle_reasoning.config as rc
    import miracle_reasoning.model as rm
    return rc, rm


def instrument(model, backend, log):
    """Wrap instance methods to capture per-step discrete decisions."""
    decisions = []
    cfg = model.config
    original_step, original_heavy, original_moe = model._step, model._heavy_attention, model._moe
    original_lighting = model._lighting

    def step(token):
        decisions.append({"topk": [], "experts": [], "expert_weights": [], "latent_positions": [],
                          "memory_size": []})
        return original_step(token)

    def heavy(x, prefix, state, position):
        before = len(backend.uploads)
        out = original_heavy(x, prefix, state, position)
        count = state["ring"].count
        length = min(cfg.window, count)
        blocks = -(-count // cfg.source["long_context"]["global_block_size"])
        # The masked score matrix is the upload of shape [heads, length+blocks]
        # (weight-cache misses upload weights during the same call).
        masked = [u for u in backend.uploads[before:] if u.shape == (cfg.query_heads, length + blocks)][-1]
        block_cols = masked[:, length:]
        decisions[-1]["topk"].append([np.flatnonzero(np.isfinite(r)).tolist() for r in block_cols])
        return out

    def moe(x, prefix):
        before = len(log)
        scales = []
        original_add = backend.add

        def add(a, b, scale=1.0):
            scales.append(float(scale))
            return original_add(a, b, scale)

        backend.add = add
        try:
            out = original_moe(x, prefix)
        finally:
            backend.add = original_add
        chosen = []
        for name in log[before:]:
            if name.startswith(prefix + "experts.") and name.endswith(".gate"):
                expert = int(name[len(prefix + "experts."):].split(".")[0])
                if expert not in chosen:  # a cache miss reads the same name twice
                    chosen.append(expert)
        decisions[-1]["experts"].append(chosen)
        decisions[-1]["expert_weights"].append(scales[:len(chosen)])
        return out

    def lighting(x, prefix, state, position):
        out = original_lighting(x, prefix, state, position)
        decisions[-1]["latent_positions"].append(list(state["positions"]))
        decisions[-1]["memory_size"].append(int(state["memory_size"]))
        return out

    model._step, model._heavy_attention, model._moe, model._lighting = step, heavy, moe, lighting
    return decisions


def state_summary(model):
    out = []
    for st in model.states:
        entry = {}
        if "ring" in st:
            r = st["ring"]
            entry["ring"] = [r.count, r.length, r.start, r.capacity]
        if "relay" in st:
            entry["relay"] = st["relay"].count
        if "latent" in st:
            entry["latent_rows"] = st["latent"].shape[0]
            entry["positions"] = list(st["positions"])
            entry["counts"] = list(st["counts"])
            entry["memory_size"] = st["memory_size"]
        if "loops" in st:
            entry["loops"] = [[s["ring"].count, s["ring"].capacity] for s in st["loops"]]
        out.append(entry)
    return out


def run_micro(name, rc, rm):
    config = cases.micro_config(name)
    ref_config = rc.ModelConfig.from_dict(config.to_dict())
    weights = cases.micro_weights(config)
    log = []
    backend = HostBackend("reference")
    backend.record_uploads = True
    model = rm.MiracleModel(ref_config, RecordingWeights(weights, log), backend=backend,
                            context_length=cases.micro_context(name))
    decisions = instrument(model, backend, log)
    prompt = cases.micro_prompt(name)
    logits = model.prefill(prompt, return_all=True)
    summary = state_summary(model)
    model.reset()
    split = 5
    chunked = np.concatenate([model.prefill(prompt[:split], return_all=True),
                              model.prefill(prompt[split:], return_all=True)])
    greedy = model.generate(prompt[:3], max_new_tokens=6)
    sampled = model.generate(prompt[:2], max_new_tokens=5, temperature=0.8, top_k=5, top_p=0.9, seed=7)
    prefill_decisions = decisions[:len(prompt)]
    np.savez_compressed(
        HERE / f"micro_{name}.npz", logits=logits.astype(np.float32), chunked=chunked.astype(np.float32),
        greedy=np.asarray(greedy, np.int64), sampled=np.asarray(sampled, np.int64),
        prompt=np.asarray(prompt, np.int64),
        meta=json.dumps({"state": summary, "decisions": prefill_decisions}))
    return logits.shape


class LazyWeights(Mapping):
    """The synthetic BF16 model of a configuration, generated tensor by tensor
    when the reference reads it (the 36B Heavy Medium model does not fit this
    host's memory at once).  Generated tensors are kept in an LRU of
    ``budget_bytes`` of BF16 bits; the values are exactly those of
    ``synthetic.synthetic_weights`` (and of the device fill kernel)."""

    def __init__(self, config, seed=0, budget_bytes=34 << 30):
        from collections import OrderedDict
        self.plan = {name: (index, shape, std) for index, name, shape, std in cases.synthetic.tensor_plan(config)}
        self.seed, self.budget, self.used, self.cache = seed, budget_bytes, 0, OrderedDict()

    def __iter__(self):
        return iter(self.plan)

    def __len__(self):
        return len(self.plan)

    def __contains__(self, key):
        return key in self.plan

    def __getitem__(self, key):
        index, shape, std = self.plan[key]
        if std is None:
            return np.ones(shape, np.float32)
        return _LazyTensor(self, key, shape)

    def bits(self, key):
        if key in self.cache:
            self.cache.move_to_end(key)
            return self.cache[key]
        index, shape, std = self.plan[key]
        data = cases.synthetic.hash_normal_bf16(self.seed, index, shape, std)
        while self.cache and self.used + data.nbytes > self.budget:
            _, old = self.cache.popitem(last=False)
            self.used -= old.nbytes
        self.cache[key] = data
        self.used += data.nbytes
        return data


class _LazyTensor:
    def __init__(self, owner, key, shape):
        self.owner, self.key, self.shape = owner, key, tuple(shape)

    def __getitem__(self, index):
        return cases.widen_bf16(self.owner.bits(self.key)[index])

    def __array__(self, dtype=None, copy=None):
        result = self[:]
        return result.astype(dtype, copy=False) if dtype is not None else result


def run_bench(name, rc, rm):
    """A BASELINE architecture at full size: the prompt, then greedy decode
    steps.  Saved per step (prompt's last token, then each decode step): the
    leading logits, every LOGIT_STRIDE-th logit (all of them for small
    vocabularies), the top 64 ids and values, the greedy ids; for Heavy
    Medium also the routed experts (with their weights) and the kept global
    blocks of every layer and inner loop."""
    config, stored, ctx, prompt, steps = cases.bench_case(name)
    ref_config = rc.ModelConfig.from_dict(config.to_dict())
    heavy = config.family == "heavy-medium-2.0"
    log = []
    weights = LazyWeights(config) if heavy else cases.synthetic.synthetic_weights(config, stored)
    backend = HostBackend("reference")
    if heavy:
        block = config.source["long_context"]["global_block_size"]
        backend.record_uploads = lambda a: a.ndim == 2 and a.shape[0] == config.query_heads and \
            a.shape[1] <= config.window + (ctx + block - 1) // block
        weights = RecordingWeights(weights, log)
    model = rm.MiracleModel(ref_config, weights, backend=backend, context_length=ctx)
    decisions = instrument(model, backend, log) if heavy else None
    t0 = time.time()
    logits = [model.prefill(prompt)]
    tokens = []
    for _ in range(steps):
        tokens.append(int(np.argmax(logits[-1])))
        logits.append(model.decode(tokens[-1]))
        print(f"  {name}: step {len(tokens)} of {steps} ({time.time() - t0:.0f} s)", flush=True)
    elapsed = time.time() - t0
    stack = np.stack(logits).astype(np.float32)
    top = np.argsort(-stack, axis=1, kind="stable")[:, :cases.TOPK_STORED]
    meta = {"context": ctx, "stored": stored, "seconds": elapsed, "tokens_processed": len(prompt) + steps}
    if heavy:  # per token (prompt and steps): kept blocks, experts, weights of every (layer, loop)
        meta["decisions"] = [{k: d[k] for k in ("topk", "experts", "expert_weights")} for d in decisions]
    np.savez_compressed(
        HERE / f"bench_{name}.npz", lead=stack[:, :cases.LOGIT_SUBSET], top_ids=top.astype(np.int64),
        top_values=np.take_along_axis(stack, top, axis=1), tokens=np.asarray(tokens, np.int64),
        prompt=np.asarray(prompt, np.int64),
        full=stack if stack.shape[1] <= 4096 else np.zeros((0,), np.float32),
        strided=stack[:, ::cases.LOGIT_STRIDE],
        meta=json.dumps(meta))
    return stack.shape, elapsed


def config_variants():
    """Configurations whose RoPE tables / name tables are pinned against the reference."""
    variants = {name: cases.micro_config(name) for name in cases.MICRO_CASES}
    for name in ("nano15", "nano17", "lite", "lighting", "heavy"):
        variants["bench_" + name] = cases.synthetic.config_for(name)
    base = cases.micro_config("lighting")
    for kind in ("linear", "dynamic_ntk", "none"):
        src = dict(base.source, rope_scaling_type=kind, rope_scaling_factor=4.0,
                   extension_max_position_embeddings=64)
        variants[f"lighting_{kind}"] = cases.replace(base, head_dim=8, hidden_size=32, source=src)
    variants["nano17_yarn"] = cases.replace(
        cases.micro_config("nano17"), head_dim=16, hidden_size=64,
        source={"rope_scaling": {"type": "yarn", "factor": 4.0, "orig_max_position": 32,
                                 "beta_fast": 32, "beta_slow": 1}})
    return variants


def run_configs(rc):
    import miracle_reasoning.weights as rw
    freqs, meta = {}, {}
    for name, config in config_variants().items():
        ref = rc.ModelConfig.from_dict(config.to_dict())
        freqs[name] = ref.inverse_frequencies()
        meta[name] = {"to_dict": json.loads(json.dumps(ref.to_dict())),
                      "native_names": rw.native_names(ref),
                      "expected_shapes": {k: list(v) for k, v in rw.expected_shapes(ref).items()}}
    np.savez_compressed(HERE / "configs.npz", **{f"freq_{k}": v for k, v in freqs.items()},
                        meta=json.dumps(meta))


def run_kernels():
    b = HostBackend("reference")
    out = {}
    rng = np.random.default_rng(9)
    x = rng.normal(size=(3, 19)).astype(np.float32)
    w = rng.normal(size=(7, 19)).astype(np.float32)
    scales = rng.normal(size=19).astype(np.float32)
    out.update(lin_x=x, lin_w=w, lin_y=b.read(b.linear(b.upload(x), b.upload(w))), rms_w=scales,
               rms_y=b.read(b.norm(b.upload(x), b.upload(scales), 19, 1e-6)))
    logits = np.array([[1000, 1001, -1000], [-1000, -1001, -1002]], np.float32)
    out.update(sm_x=logits, sm_y=b.read(b.softmax(b.upload(logits))))
    rng = np.random.default_rng(3)
    rx = rng.normal(size=(2, 3, 6)).astype(np.float32)
    pos, freq = np.array([7, 29], np.float32), np.array([1, .1, .01], np.float32)
    out["rope_x"] = rx
    for split in (0, 1):
        out[f"rope_y{split}"] = b.read(b.rotate(b.upload(rx.reshape(2, 18)), b.upload(freq), b.upload(pos), 3, 6,
                                                bool(split)))
    rng = np.random.default_rng(6)
    q = rng.normal(size=(4, 6)).astype(np.float32)
    k, v = [rng.normal(size=(5, 2, 6)).astype(np.float32) for _ in range(2)]
    rk, rv = [rng.normal(size=(3, 2, 6)).astype(np.float32) for _ in range(2)]
    att = b.attention(b.upload(q.reshape(1, -1)), b.upload(k.reshape(5, -1)), b.upload(v.reshape(5, -1)),
                      heads=4, kv_heads=2, dim=6, start=3, length=4, extra_keys=b.upload(rk.reshape(3, -1)),
                      extra_values=b.upload(rv.reshape(3, -1)), extra_length=3)
    out.update(att_q=q, att_k=k, att_v=v, att_rk=rk, att_rv=rv, att_y=b.read(att))
    np.savez_compressed(HERE / "kernels.npz", **out)


def run_prefill(name, rc, rm):
    """BF16 micro model: all-token logits of a 48-token prompt, the same prompt
    in two chunks, and greedy decode steps after it (the reference widens
    BF16 exactly, so it runs on the widened values)."""
    config = cases.prefill_config(name)
    ref_config = rc.ModelConfig.from_dict(config.to_dict())
    weights = {k: (cases.widen_bf16(v) if v.dtype == np.uint16 else v)
               for k, v in cases.prefill_weights(config).items()}
    model = rm.MiracleModel(ref_config, weights, backend=HostBackend("reference"),
                            context_length=cases.PREFILL_CONTEXT)
    prompt = cases.prefill_prompt(name)
    logits = model.prefill(prompt, return_all=True)
    summary = state_summary(model)
    steps, tokens = [], []
    for _ in range(4):
        tokens.append(int(np.argmax(steps[-1] if steps else logits[-1])))
        steps.append(model.decode(tokens[-1]))
    model.reset()
    split = cases.PREFILL_SPLIT
    chunked = np.concatenate([model.prefill(prompt[:split], return_all=True),
                              model.prefill(prompt[split:], return_all=True)])
    np.savez_compressed(
        HERE / f"prefill_{name}.npz", logits=logits.astype(np.float32), chunked=chunked.astype(np.float32),
        steps=np.stack(steps).astype(np.float32), tokens=np.asarray(tokens, np.int64),
        prompt=np.asarray(prompt, np.int64), meta=json.dumps({"state": summary}))
    return logits.shape


def main(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", type=Path, default=os.environ.get("MIRACLE_REFERENCE_ROOT"),
                        help="the reference checkout (default: $MIRACLE_REFERENCE_ROOT)")
    parser.add_argument("--only", nargs="*")
    args = parser.parse_args(argv)
    if args.reference_root is None:
        parser.error("--reference-root (or MIRACLE_REFERENCE_ROOT) is required")
    rc, rm = _ref_modules(args.reference_root)
    todo = args.only or ["kernels", "configs", *[f"micro_{c}" for c in cases.MICRO_CASES],
                         *[f"bench_{c}" for c in cases.BENCH_CASES],
                         *[f"prefill_{c}" for c in cases.PREFILL_CASES]]
    for item in todo:
        t0 = time.time()
        if item == "kernels":
            run_kernels()
            result = "ok"
        elif item == "configs":
            run_configs(rc)
            result = "ok"
        elif item.startswith("micro_"):
            result = run_micro(item[6:], rc, rm)
        elif item.startswith("prefill_"):
            result = run_prefill(item[8:], rc, rm)
        else:
            result = run_bench(item[6:], rc, rm)
        print(f"{item}: {result} ({time.time() - t0:.1f}s)", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
