"""One rank of the tensor- / expert-parallel decode check (launched by
tests/test_gpu_tp.py under torch.distributed.run, one process per GPU).

Rank 0 first runs the prompt and greedy decode steps on a single-GPU model;
then every rank builds the same model split over the ranks and repeats them.
Rank 0 writes the comparison (greedy ids, largest logit difference) as JSON.
"""
from __future__ import annotations

import datetime
import importlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
PKG = "miraclereasoning-cpu_b200"
syn = importlib.import_module(PKG + ".synthetic")
MiracleModel = importlib.import_module(PKG + ".model").MiracleModel
CUDABackend = importlib.import_module(PKG + ".backend").CUDABackend


def small_heavy():
    """Heavy Medium at test size: 16 routed experts (8 per rank at 2 ranks), 2 shared."""
    return importlib.import_module(PKG + ".config").ModelConfig(
        family="heavy-medium-2.0", vocab_size=512, hidden_size=256, layers=2, query_heads=4, kv_heads=2,
        head_dim=64, ffn_dim=128, max_positions=2048, window=32, latent_dim=64, inner_loop_steps=2,
        source={"routed_experts": 16, "router_groups": 4, "router_top_k_max": 4, "router_top_k_min": 2,
                "shared_experts": 2,
                "long_context": {"local_window": 32, "global_block_size": 8, "global_slots": 3,
                                 "target_context": 2048}})


def run(model, prompt, steps):
    logits = [model.prefill(prompt)]
    tokens = []
    for _ in range(steps):
        tokens.append(int(np.argmax(logits[-1])))
        logits.append(model.decode(tokens[-1]))
    return tokens, np.stack(logits)


def run_failure(out_path, rank, world, backend, all_gather):
    """Rank 1 stays alive but skips one decode call: rank 0's step waits for
    rank 1's exchange words, its bounded wait runs out (200 ms) and the call
    raises; then the ranks tear down in order (a barrier before and after the
    models are released, so no rank frees its arena while a peer's kernel
    could still store into it)."""
    import gc
    import time
    native = importlib.import_module(PKG + "._native")
    config = syn.config_for("nano17")
    model = MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=256,
                                   tensor_parallel=(rank, world, all_gather))
    native.call("mr_model_set_wait_limit", model._handle, 200_000_000)
    prompt = syn.prompt_ids(config.vocab_size, 8, seed=3).tolist()
    token = int(np.argmax(model.prefill(prompt)))
    token = int(np.argmax(model.decode(token)))  # one step together
    dist.barrier()
    outcome = {"rank1_skipped": True}
    if rank == 0:
        t0 = time.perf_counter()
        try:
            model.decode(token)
            outcome.update(code=0, message="no error")
        except native.CUDAError as exc:
            outcome.update(code=exc.code, message=str(exc))
        outcome["seconds"] = time.perf_counter() - t0
        try:
            model.decode(token)
        except RuntimeError as exc:
            outcome["latched"] = "reset" in str(exc)
    dist.barrier()  # tear down in order
    del model
    gc.collect()
    dist.barrier()
    if rank == 0:
        Path(out_path).write_text(json.dumps(outcome))
    dist.destroy_process_group()


def main():
    out_path, config_name, steps = sys.argv[1], sys.argv[2], int(sys.argv[3])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    backend = CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    if config_name == "fail":
        def gather(data):
            items = [None] * world
            dist.all_gather_object(items, data)
            return items
        return run_failure(out_path, rank, world, backend, gather)
    config = small_heavy() if config_name == "heavy_small" else syn.config_for(config_name)
    prompt = syn.prompt_ids(config.vocab_size, 40, seed=3).tolist()
    context = 1024
    if rank == 0:
        single = MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=context)
        if config_name == "heavy_small":
            # expert parallel runs prompts through the token step: so does the reference run,
            # which makes the two comparable bit for bit
            importlib.import_module(PKG + "._native").call("mr_model_set_batched_prefill", single._handle, 0, None)
        ref_tokens, ref_logits = run(single, prompt, steps)
        del single
    dist.barrier()

    def all_gather(data):
        items = [None] * world
        dist.all_gather_object(items, data)
        return items

    model = MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=context,
                                   tensor_parallel=(rank, world, all_gather))
    dist.barrier()
    tokens, logits = run(model, prompt, steps)
    dist.barrier()
    if rank == 0:
        scale = float(np.abs(ref_logits).max())
        result = {"tokens": tokens, "ref_tokens": ref_tokens,
                  "max_abs_diff": float(np.abs(logits - ref_logits).max()), "scale": scale,
                  "ranks": world}
        Path(out_path).write_text(json.dumps(result))
    del model
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
