"""The command line (miraclereasoning-cpu_b200/cli.py), the reference's
`devices` / `generate` commands on the CUDA backend (cli.py:30-91)."""
import json
import subprocess
import sys

import numpy as np
import pytest

import cases
from conftest import REPO, submodule

CLI = REPO / "miraclereasoning-cpu_b200" / "cli.py"


def _run(*args):
    return subprocess.run([sys.executable, str(CLI), *args], capture_output=True, text=True, timeout=300)


def test_cli_parses_the_reference_arguments():
    cli = submodule("cli")
    args = cli.build_parser().parse_args(["generate", "m", "--ids", "1,2 3", "--max-new-tokens", "4",
                                          "--temperature", "0.5", "--top-k", "3", "--top-p", "0.9", "--seed", "5"])
    assert (args.command, args.ids, args.max_new_tokens, args.top_k, args.seed) == ("generate", "1,2 3", 4, 3, 5)
    with pytest.raises(SystemExit):
        cli.build_parser().parse_args(["generate", "m"])  # --ids or --prompt is required


def test_cli_errors_exit_2_with_a_message(tmp_path):
    done = _run("generate", str(tmp_path), "--prompt", "hello")
    assert done.returncode == 2 and done.stderr.startswith("error: --prompt requires --tokenizer")


@pytest.mark.gpu
def test_cli_generate_matches_the_model(tmp_path):
    config = cases.micro_config("nano15")
    weights = cases.micro_weights(config)
    (tmp_path / "config.json").write_text(json.dumps(config.to_dict()))
    np.savez(tmp_path / "model.npz", **weights)
    done = _run("generate", str(tmp_path), "--ids", "1 5 3", "--max-new-tokens", "6", "--context-length", "16")
    assert done.returncode == 0, done.stderr
    out = json.loads(done.stdout)
    model = submodule("model").MiracleModel(config, weights, backend=submodule("backend").CUDABackend(),
                                            context_length=16)
    assert out["token_ids"] == model.generate([1, 5, 3], max_new_tokens=6)
    sampled = _run("generate", str(tmp_path), "--ids", "1,5", "--max-new-tokens", "5", "--temperature", "0.8",
                   "--top-k", "5", "--top-p", "0.9", "--seed", "7", "--context-length", "16")
    assert json.loads(sampled.stdout)["token_ids"] == model.generate([1, 5], max_new_tokens=5, temperature=0.8,
                                                                     top_k=5, top_p=0.9, seed=7)
