"""Tensor-parallel decode (every projection and the lm_head split by output row
over the GPUs, attention by KV head, exchange words stored into every rank's
arena over NVLink) and Heavy Medium expert-parallel decode (experts by id
modulo ranks, expert rows stored into every rank's arena) against the
single-GPU engine on the same model and prompt.

Runs tests/tp_worker.py as one process per GPU under torch.distributed.run
(127.0.0.1 rendezvous); a case is skipped when the box has fewer GPUs than it
has ranks.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def _gpus():
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=30).stdout
    except (OSError, subprocess.TimeoutExpired):
        return 0
    return sum(1 for line in out.splitlines() if line.startswith("GPU "))


GPUS = _gpus()


# 8 ranks over nano-1.7's 4 local KV heads: half the ranks hold no head of those layers;
# heavy_small: Heavy Medium expert parallel (experts by id modulo ranks)
@pytest.mark.parametrize("config,ranks", [("nano17", 2), ("lite", 2), ("lighting", 2), ("heavy_small", 2),
                                          ("nano17", 4), ("heavy_small", 4), ("nano17", 8)])
def test_tensor_parallel_decode_matches_single_gpu(tmp_path, config, ranks):
    if GPUS < ranks:
        pytest.skip(f"tensor-parallel decode over {ranks} GPUs needs {ranks} GPUs")
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(ranks), "--master-addr", "127.0.0.1", "--master-port", str(29500 + 17 * ranks),
           str(REPO / "tests" / "tp_worker.py"), str(out), config, "6"]
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=420)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    result = json.loads(out.read_text())
    assert result["tokens"] == result["ref_tokens"]
    # both sum every dot product in the same order per row: the split only moves rows between GPUs
    assert result["max_abs_diff"] <= 2e-5 * max(1.0, result["scale"])
    if config == "heavy_small":  # the same kernels compute each expert, wherever it runs
        assert result["max_abs_diff"] == 0.0


def test_a_rank_that_skips_a_step_makes_the_other_time_out(tmp_path):
    """Two ranks decode one sequence; rank 1 stays alive but skips one decode
    call.  Rank 0's bounded waits for rank 1's words run out: its call raises
    MR_ERR_TIMEOUT quickly, the model latches until reset(), and both ranks
    release their models in order and exit cleanly (tests/tp_worker.py
    run_failure).  No GPU is faulted; NVLS is off."""
    if GPUS < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "fail.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29611",
           str(REPO / "tests" / "tp_worker.py"), str(out), "fail", "0"]
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=420)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    result = json.loads(out.read_text())
    assert result["code"] == 4, result  # MR_ERR_TIMEOUT
    assert result["seconds"] < 30.0 and result["latched"], result
