#!/usr/bin/env python3
"""Exact-tokenization text frontend over the B200 `qwen3` program.

    python -m xpu_playground_b200.chat --model-dir DIR --prompt TEXT
        --max-new-tokens N [--system TEXT] [--max-seq-len N]
        [--thinking | --no-thinking]

The same command line, checks, exit codes and output as the reference's
frontend (qwen3/chat.py:10-96): the prompt is rendered with the checkpoint's
own chat template (transformers' AutoTokenizer, local files only, no remote
code), the token ids go to the native engine on standard input
(`--input-ids -`, one space-separated line; qwen3/main.cpp:331-358), the
engine answers one JSON line `{"generated_ids":[...]}` and the generated ids
are decoded with special tokens kept and written to standard output.

The engine is this package's `qwen3` program (xpu_playground_b200/bin/qwen3,
built by xpu_playground_b200.build), which decodes on the GPU; the frontend
itself only tokenizes and decodes text on the host.
"""

from __future__ import annotations

import argparse
import json
import subprocess
import sys
from pathlib import Path

MAX_SEQUENCE = 40960  # qwen3/chat.py:28-29, qwen3/main.cpp kMaximumContext
DEFAULT_ENGINE = Path(__file__).resolve().parent / "bin" / "qwen3"


def parse_args(argv=None) -> argparse.Namespace:
    """Flags of qwen3/chat.py:10-32, with the engine defaulting to this
    package's `qwen3` program."""
    parser = argparse.ArgumentParser(description="Greedy single-turn Qwen3 chat on B200")
    parser.add_argument("--model-dir", required=True, type=Path)
    parser.add_argument("--prompt", required=True)
    parser.add_argument("--system")
    parser.add_argument("--max-new-tokens", type=int, required=True)
    parser.add_argument("--max-seq-len", type=int, default=MAX_SEQUENCE)
    thinking = parser.add_mutually_exclusive_group()
    thinking.add_argument("--thinking", action="store_true", dest="thinking")
    thinking.add_argument("--no-thinking", action="store_false", dest="thinking")
    parser.set_defaults(thinking=False)
    parser.add_argument("--engine", type=Path, default=DEFAULT_ENGINE, help=argparse.SUPPRESS)
    args = parser.parse_args(argv)
    if args.max_new_tokens < 0:
        parser.error("--max-new-tokens must be non-negative")
    if not 1 <= args.max_seq_len <= MAX_SEQUENCE:
        parser.error(f"--max-seq-len must be in [1, {MAX_SEQUENCE}]")
    return args


def prompt_ids(tokenizer, prompt: str, system: str | None, thinking: bool) -> list[int]:
    """The chat-templated prompt as token ids (qwen3/chat.py:50-60).

    transformers 4.x returns a list from apply_chat_template(tokenize=True);
    5.x returns a BatchEncoding whose "input_ids" holds the same list."""
    messages = []
    if system is not None:
        messages.append({"role": "system", "content": system})
    messages.append({"role": "user", "content": prompt})
    ids = tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=True,
                                        enable_thinking=thinking)
    if not isinstance(ids, list):
        ids = ids["input_ids"]
    return [int(i) for i in ids]


def run_engine(engine: Path, model_dir: Path, ids: list[int], max_new_tokens: int,
               max_seq_len: int) -> list[int]:
    """Runs the native engine with the ids on standard input and parses its
    JSON answer (qwen3/chat.py:72-93). Raises CalledProcessError when the
    engine fails and ValueError when its output is not the expected JSON."""
    command = [str(engine), "--model-dir", str(model_dir), "--input-ids", "-",
               "--max-new-tokens", str(max_new_tokens), "--max-seq-len", str(max_seq_len)]
    completed = subprocess.run(command, input=" ".join(map(str, ids)) + "\n", text=True,
                               stdout=subprocess.PIPE, check=True)
    payload = json.loads(completed.stdout)
    generated = payload["generated_ids"]
    if not isinstance(generated, list) or not all(isinstance(i, int) for i in generated):
        raise ValueError("generated_ids is not an integer list")
    return generated


def main(argv=None) -> int:
    args = parse_args(argv)
    try:
        from transformers import AutoTokenizer
    except ImportError:
        print("qwen3 chat: transformers is required for the tokenizer", file=sys.stderr)
        return 1
    # local_files_only: the model directory is the only source of the tokenizer.
    tokenizer = AutoTokenizer.from_pretrained(args.model_dir, local_files_only=True,
                                              trust_remote_code=False)
    input_ids = prompt_ids(tokenizer, args.prompt, args.system, args.thinking)
    if len(input_ids) + args.max_new_tokens > args.max_seq_len:
        print(f"qwen3 chat: tokenized request needs {len(input_ids) + args.max_new_tokens} "
              f"positions but --max-seq-len is {args.max_seq_len}", file=sys.stderr)
        return 1
    if not args.engine.is_file():
        print(f"qwen3 chat: native engine not found: {args.engine}; "
              "run 'python -m xpu_playground_b200.build'", file=sys.stderr)
        return 1
    try:
        generated = run_engine(args.engine, args.model_dir, input_ids, args.max_new_tokens,
                               args.max_seq_len)
    except subprocess.CalledProcessError as error:
        return error.returncode or 1
    except (json.JSONDecodeError, KeyError, ValueError) as error:
        print(f"qwen3 chat: invalid native-engine output: {error}", file=sys.stderr)
        return 1
    sys.stdout.write(tokenizer.decode(generated, skip_special_tokens=False))
    sys.stdout.flush()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
