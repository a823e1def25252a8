"""Command line of the CUDA engine.

    python miraclereasoning-cpu_b200/cli.py devices
    python miraclereasoning-cpu_b200/cli.py generate MODEL_DIR --ids "1 5 73" [--max-new-tokens 32]
        [--temperature T --top-k K --top-p P --seed S] [--context-length N] [--device-index I]
    python miraclereasoning-cpu_b200/cli.py generate MODEL_DIR --prompt TEXT --tokenizer TOK.model
    python miraclereasoning-cpu_b200/cli.py inspect MODEL_DIR

The interface is the reference's (miracle_reasoning/cli.py:30-91): the same
sub-commands, flags and JSON keys (`device`, `token_ids`, `text`; for
`inspect` the model summary), and `error: ...` on stderr with exit status 2
for a bad request.  Generation runs on a B200 through `CUDABackend` and
`MiracleModel`; the reference's `export` (PyTorch checkpoint conversion) is
host tooling with no device work and is not repeated here.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import sys
from dataclasses import dataclass
from pathlib import Path

if __package__ in (None, ""):  # run as a script: import the package by its directory name
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    _pkg = importlib.import_module(Path(__file__).resolve().parent.name)
else:
    _pkg = importlib.import_module(__package__)

# What a request can get wrong, reported as `error: ...` with exit status 2.
_REQUEST_ERRORS = (ValueError, OSError, KeyError, ImportError, RuntimeError, FloatingPointError)


class TextCodec:
    """Text <-> token ids through a SentencePiece model (.model) or, when the
    `tokenizers` package is installed, a tokenizer.json; no special tokens are
    added, as in the reference."""

    def __init__(self, path: Path):
        path = Path(path)
        if path.suffix == ".model":
            import sentencepiece
            processor = sentencepiece.SentencePieceProcessor(model_file=str(path))
            self._encode, self._decode = processor.encode, processor.decode
        else:
            from tokenizers import Tokenizer
            tokenizer = Tokenizer.from_file(str(path))
            self._encode = lambda text: tokenizer.encode(text, add_special_tokens=False).ids
            self._decode = tokenizer.decode

    def encode(self, text: str) -> list[int]:
        return list(self._encode(text))

    def decode(self, ids) -> str:
        return self._decode(list(ids))


@dataclass
class GenerateRequest:
    model_dir: Path
    ids: list[int]
    codec: TextCodec | None
    family: str | None
    context_length: int | None
    weight_cache_bytes: int
    device_index: int
    sampling: dict

    @classmethod
    def from_args(cls, args) -> "GenerateRequest":
        codec = None
        if args.prompt is not None:
            if args.tokenizer is None:
                raise ValueError("--prompt requires --tokenizer (SentencePiece .model or tokenizers .json)")
            codec = TextCodec(args.tokenizer)
            ids = codec.encode(args.prompt)
        else:
            ids = [int(field) for field in args.ids.replace(",", " ").split()]
        sampling = {"max_new_tokens": args.max_new_tokens, "temperature": args.temperature, "top_k": args.top_k,
                    "top_p": args.top_p, "seed": args.seed}
        return cls(args.model_dir, ids, codec, args.family, args.context_length, args.weight_cache_mib << 20,
                   args.device_index, sampling)


def cmd_devices(args) -> dict | list:
    return [device.to_dict() for device in _pkg.list_devices()]


def cmd_inspect(args) -> dict:
    config = _pkg.ModelConfig.from_dict(json.loads((args.model_dir / "config.json").read_text(encoding="utf-8")),
                                        args.family)
    shapes = importlib.import_module(_pkg.__name__ + ".weights").expected_shapes(config)
    parameters = sum(math.prod(shape) for shape in shapes.values())
    return {"family": config.family, "layers": config.layers, "hidden_size": config.hidden_size,
            "max_positions": config.max_positions, "inference_parameters": parameters,
            "fp32_weight_bytes": parameters * 4}


def cmd_generate(args) -> dict:
    request = GenerateRequest.from_args(args)
    backend = _pkg.CUDABackend(device_index=request.device_index)
    model = _pkg.MiracleModel.from_pretrained(request.model_dir, family=request.family, backend=backend,
                                              context_length=request.context_length,
                                              weight_cache_bytes=request.weight_cache_bytes)
    tokens = model.generate(request.ids, **request.sampling)
    result = {"device": backend.device.to_dict(), "token_ids": tokens}
    if request.codec is not None:
        result["text"] = request.codec.decode(tokens)
    return result


COMMANDS = {"devices": cmd_devices, "inspect": cmd_inspect, "generate": cmd_generate}


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description="MiracleReasoning token loop on NVIDIA B200 (CUDA)")
    commands = parser.add_subparsers(dest="command", required=True)
    commands.add_parser("devices", help="list CUDA devices and their memory limits")
    inspect = commands.add_parser("inspect", help="summarise a model directory's configuration")
    inspect.add_argument("model_dir", type=Path)
    inspect.add_argument("--family", choices=_pkg.FAMILIES)
    generate = commands.add_parser("generate", help="generate tokens on a CUDA device")
    generate.add_argument("model_dir", type=Path)
    source = generate.add_mutually_exclusive_group(required=True)
    source.add_argument("--ids", help="comma/space separated token IDs")
    source.add_argument("--prompt")
    generate.add_argument("--tokenizer", type=Path)
    generate.add_argument("--family", choices=_pkg.FAMILIES)
    generate.add_argument("--context-length", type=int, help="default: min(2048, model context limit)")
    generate.add_argument("--weight-cache-mib", type=int, default=256,
                          help="kept for the reference's interface; the whole model is resident in HBM")
    generate.add_argument("--device-index", type=int, default=0)
    for flag, kind, default in (("--max-new-tokens", int, 32), ("--temperature", float, 0.0), ("--top-k", int, 0),
                                ("--top-p", float, 1.0), ("--seed", int, 17)):
        generate.add_argument(flag, type=kind, default=default)
    return parser


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    try:
        result = COMMANDS[args.command](args)
    except _REQUEST_ERRORS as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 2
    pretty = args.command != "generate"
    print(json.dumps(result, indent=2 if pretty else None, ensure_ascii=False))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
