"""The chat frontend (qwen3/chat.py's flags, checks and engine protocol) on
the CPU, with a stand-in engine: a script that records the command line and
standard input it was given and answers like qwen3/main.cpp:353-358."""

import json
import subprocess
import sys
import textwrap

import pytest

from tests._tokenizer import write_tokenizer
from xpu_playground_b200 import chat

FAKE_ENGINE = textwrap.dedent("""\
    #!{python}
    import json, sys
    ids = sys.stdin.read()
    with open({log!r}, "w") as f:
        json.dump({{"argv": sys.argv[1:], "stdin": ids}}, f)
    mode = {mode!r}
    if mode == "fail":
        sys.exit(3)
    if mode == "garbage":
        print("not json")
    elif mode == "floats":
        print(json.dumps({{"generated_ids": [1.5, 2]}}))
    else:
        print(json.dumps({{"generated_ids": [4, 5, 6, {end}]}}))
""")


@pytest.fixture
def model_dir(tmp_path):
    d = tmp_path / "model"
    d.mkdir()
    specials = write_tokenizer(d, 64)
    return d, specials


def fake_engine(tmp_path, mode, end):
    path = tmp_path / f"engine_{mode}"
    log = tmp_path / f"engine_{mode}.json"
    path.write_text(FAKE_ENGINE.format(python=sys.executable, log=str(log), mode=mode, end=end))
    path.chmod(0o755)
    return path, log


class Result:
    def __init__(self, returncode, stdout, stderr):
        self.returncode, self.stdout, self.stderr = returncode, stdout, stderr


@pytest.fixture
def run_chat(capsys):
    """chat.main in this process (transformers is imported once), with its
    exit status, standard output and standard error."""
    def run(*args):
        capsys.readouterr()
        try:
            code = chat.main([str(a) for a in args])
        except SystemExit as e:  # argparse errors
            code = e.code
        out = capsys.readouterr()
        return Result(code, out.out, out.err)
    return run


def test_module_runs_as_a_program(tmp_path, model_dir):
    d, sp = model_dir
    engine, _ = fake_engine(tmp_path, "ok", sp["<|im_end|>"])
    r = subprocess.run([sys.executable, "-m", "xpu_playground_b200.chat", "--model-dir", str(d), "--prompt", "w1",
                        "--max-new-tokens", "3", "--engine", str(engine)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout == "w4 w5 w6 <|im_end|>"


def test_chat_sends_template_ids_and_decodes_the_answer(tmp_path, model_dir, run_chat):
    d, sp = model_dir
    engine, log = fake_engine(tmp_path, "ok", sp["<|im_end|>"])
    r = run_chat("--model-dir", d, "--prompt", "w1 w2 w3", "--system", "w9",
                 "--max-new-tokens", 7, "--max-seq-len", 100, "--engine", engine)
    assert r.returncode == 0, r.stderr
    assert r.stdout == "w4 w5 w6 <|im_end|>"
    seen = json.loads(log.read_text())
    assert seen["argv"] == ["--model-dir", str(d), "--input-ids", "-", "--max-new-tokens", "7",
                            "--max-seq-len", "100"]
    expected = [sp["<|im_start|>"], sp["system"], 9, sp["<|im_end|>"],
                sp["<|im_start|>"], sp["user"], 1, 2, 3, sp["<|im_end|>"],
                sp["<|im_start|>"], sp["assistant"], sp["<think>"], sp["</think>"]]
    assert seen["stdin"] == " ".join(map(str, expected)) + "\n"


def test_chat_thinking_flag_reaches_the_template(tmp_path, model_dir, run_chat):
    d, sp = model_dir
    engine, log = fake_engine(tmp_path, "ok", sp["<|im_end|>"])
    r = run_chat("--model-dir", d, "--prompt", "w1", "--max-new-tokens", 1, "--thinking", "--engine", engine)
    assert r.returncode == 0, r.stderr
    ids = list(map(int, json.loads(log.read_text())["stdin"].split()))
    assert ids[-2:] == [sp["<|im_start|>"], sp["assistant"]]
    assert json.loads(log.read_text())["argv"][-1] == "40960"


def test_chat_rejects_bad_arguments_and_long_requests(tmp_path, model_dir, run_chat):
    d, sp = model_dir
    engine, _ = fake_engine(tmp_path, "ok", sp["<|im_end|>"])
    for extra in (["--max-new-tokens", "-1"], ["--max-new-tokens", "1", "--max-seq-len", "0"],
                  ["--max-new-tokens", "1", "--max-seq-len", "40961"],
                  ["--max-new-tokens", "1", "--thinking", "--no-thinking"]):
        r = run_chat("--model-dir", d, "--prompt", "w1", *extra, "--engine", engine)
        assert r.returncode == 2, extra
    # 9 template ids + 5 new tokens > 12 positions
    r = run_chat("--model-dir", d, "--prompt", "w1 w2", "--max-new-tokens", 5, "--max-seq-len", 12,
                 "--engine", engine)
    assert r.returncode == 1
    assert "needs 14 positions but --max-seq-len is 12" in r.stderr
    r = run_chat("--model-dir", d, "--prompt", "w1", "--max-new-tokens", 1, "--engine", tmp_path / "absent")
    assert r.returncode == 1 and "native engine not found" in r.stderr


@pytest.mark.parametrize("mode,code,text", [("fail", 3, ""), ("garbage", 1, "invalid native-engine output"),
                                            ("floats", 1, "not an integer list")])
def test_chat_engine_failures(tmp_path, model_dir, run_chat, mode, code, text):
    d, sp = model_dir
    engine, _ = fake_engine(tmp_path, mode, sp["<|im_end|>"])
    r = run_chat("--model-dir", d, "--prompt", "w1", "--max-new-tokens", 2, "--engine", engine)
    assert r.returncode == code
    assert text in r.stderr


def test_default_engine_is_the_package_program():
    assert chat.DEFAULT_ENGINE.name == "qwen3" and chat.DEFAULT_ENGINE.parent.name == "bin"
