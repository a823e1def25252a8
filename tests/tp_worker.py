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


def main():
    out_path, config_name, steps = sys.argv[1], sys.argv[2], int(sys.argv[3])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    backend = CUDABackend(device_index=int(os.environ.get("LOCAL_RANK", "0")))
    config = small_heavy() if config_name == "heavy_small" else syn.config_for(config_name)
    prompt = syn.prompt_ids(config.vocab_size, 40, seed=3).tolist()
    context = 1024
    if rank == 0:
        single = MiracleModel.synthetic(config, stored="BF16", backend=backend, context_length=context)
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
