"""Host logic of the ctypes twins of scripts/benchmark.py and scripts/chat.py
(CPU), and one short run of each through libq3b200.so (GPU)."""
import io
import json

import numpy as np
import pytest

from q3b200 import benchmark as bm
from q3b200 import chat


def test_trim_eos_matches_reference_rule():
    # scripts/benchmark.py:77-79: cut at the first end-of-text token
    assert bm.trim_eos([5, 6, bm.EOS_TOKEN, 7, bm.EOS_TOKEN]) == [5, 6]
    assert bm.trim_eos([bm.EOS_TOKEN]) == []
    assert bm.trim_eos(np.array([1, 2, 3])) == [1, 2, 3]


def test_synthetic_prompts_seeded_and_in_vocab():
    a, b = bm.synthetic_prompts(seed=3), bm.synthetic_prompts(seed=3)
    assert a == b and len(a) == 10
    assert [len(p) for p in a] == sorted(len(p) for p in a)
    assert all(0 <= t < bm.VOCAB for p in a for t in p)
    assert bm.synthetic_prompts(seed=4) != a
    fixed = bm.synthetic_prompts(2, seed=3, length=5)
    assert [len(p) for p in fixed] == [5, 5]


def test_prompts_file_and_id_parsing(tmp_path):
    f = tmp_path / "p.txt"
    f.write_text("1 2 3\n\n4,5, 6\n")
    assert bm.read_prompts_file(str(f)) == [[1, 2, 3], [4, 5, 6]]
    assert chat.parse_ids(" 7, 8 9 ") == [7, 8, 9]
    assert chat.encode_line("10 11", None) == [10, 11]
    with pytest.raises(ValueError):
        chat.encode_line("hello", None)


def test_chat_template_is_the_references():
    # scripts/chat.py:112 / scripts/benchmark.py:54
    assert bm.CHAT_TEMPLATE.format("hi") == "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"


@pytest.mark.gpu
def test_benchmark_twin_runs(gpu, tmp_path, capsys):
    pf = tmp_path / "p.txt"
    pf.write_text("1 2 3 4 5 6 7 8\n9 10 11 12\n")
    out = tmp_path / "r.json"
    assert bm.main(["--prompts-file", str(pf), "--max-tokens", "8", "--json", str(out)]) == 0
    r = json.load(open(out))["libq3b200"]
    assert len(r["tps"]) == 2 and all(v > 0 for v in r["tps"])
    assert "mean=" in capsys.readouterr().out


@pytest.mark.gpu
def test_chat_twin_runs(gpu, monkeypatch, capsys):
    lines = iter(["1 2 3", "", "not ids", "quit"])
    monkeypatch.setattr("builtins.input", lambda prompt="": next(lines))
    assert chat.main(["--max-tokens", "6"]) == 0
    text = capsys.readouterr().out
    assert "tok/s]" in text and "expected token ids" in text
