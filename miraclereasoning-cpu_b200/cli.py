"""Command line for the CUDA engine, mirroring the reference's `devices` and
`generate` commands (miracle_reasoning/cli.py:30-91) with the OpenCL backend
replaced by the B200 one:

    python miraclereasoning-cpu_b200/cli.py devices
    python miraclereasoning-cpu_b200/cli.py generate MODEL_DIR --ids "1 5 73" [--max-new-tokens 32]
        [--temperature T --top-k K --top-p P --seed S] [--context-length N] [--device-index I]
    python miraclereasoning-cpu_b200/cli.py generate MODEL_DIR --prompt TEXT --tokenizer TOK.model

Output is the reference's JSON (`device`, `token_ids`, and `text` with a
tokenizer); errors print `error: ...` and exit 2, as the reference does.
`inspect` and `export` are the reference's own host-only tools and stay there.
"""
from __future__ import annotations

import argparse
import importlib
import json
import sys
from pathlib import Path

if __package__ in (None, ""):  # run as a script: import the package by its directory name
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    _pkg = importlib.import_module(Path(__file__).resolve().parent.name)
else:
    _pkg = importlib.import_module(__package__)


def _tokenizer(path):
    """SentencePiece .model, or a tokenizers .json when that package is installed."""
    path = Path(path)
    if path.suffix == ".model":
        import sentencepiece
        return sentencepiece.SentencePieceProcessor(model_file=str(path))
    from tokenizers import Tokenizer
    tokenizer = Tokenizer.from_file(str(path))

    class Adapter:
        def encode(self, text):
            return tokenizer.encode(text, add_special_tokens=False).ids

        def decode(self, ids):
            return tokenizer.decode(ids)
    return Adapter()


def build_parser():
    parser = argparse.ArgumentParser(description="MiracleReasoning token loop on NVIDIA B200 (CUDA)")
    commands = parser.add_subparsers(dest="command", required=True)
    commands.add_parser("devices", help="list CUDA devices and memory limits")
    generate = commands.add_parser("generate", help="generate tokens on a CUDA device")
    generate.add_argument("model_dir", type=Path)
    inputs = generate.add_mutually_exclusive_group(required=True)
    inputs.add_argument("--ids", help="comma/space separated token IDs")
    inputs.add_argument("--prompt")
    generate.add_argument("--tokenizer", type=Path)
    generate.add_argument("--family", choices=_pkg.FAMILIES)
    generate.add_argument("--context-length", type=int, help="default: min(2048, model context limit)")
    generate.add_argument("--weight-cache-mib", type=int, default=256,
                          help="accepted for the reference's interface; the whole model is resident in HBM")
    generate.add_argument("--device-index", type=int, default=0)
    generate.add_argument("--max-new-tokens", type=int, default=32)
    generate.add_argument("--temperature", type=float, default=0.0)
    generate.add_argument("--top-k", type=int, default=0)
    generate.add_argument("--top-p", type=float, default=1.0)
    generate.add_argument("--seed", type=int, default=17)
    return parser


def main(argv=None):
    args = build_parser().parse_args(argv)
    try:
        if args.command == "devices":
            print(json.dumps([d.to_dict() for d in _pkg.list_devices()], indent=2, ensure_ascii=False))
            return 0
        tokenizer = None
        if args.prompt is not None:
            if args.tokenizer is None:
                raise ValueError("--prompt requires --tokenizer (SentencePiece .model or tokenizers .json)")
            tokenizer = _tokenizer(args.tokenizer)
            ids = tokenizer.encode(args.prompt)
        else:
            ids = [int(t) for t in args.ids.replace(",", " ").split()]
        backend = _pkg.CUDABackend(device_index=args.device_index)
        model = _pkg.MiracleModel.from_pretrained(args.model_dir, family=args.family, backend=backend,
                                                  context_length=args.context_length,
                                                  weight_cache_bytes=args.weight_cache_mib * 1024 * 1024)
        generated = model.generate(ids, max_new_tokens=args.max_new_tokens, temperature=args.temperature,
                                   top_k=args.top_k, top_p=args.top_p, seed=args.seed)
        result = {"device": backend.device.to_dict(), "token_ids": generated}
        if tokenizer:
            result["text"] = tokenizer.decode(generated)
        print(json.dumps(result, ensure_ascii=False))
        return 0
    except (ValueError, OSError, KeyError, ImportError, RuntimeError, FloatingPointError) as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 2


if __name__ == "__main__":
    raise SystemExit(main())
