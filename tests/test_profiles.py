"""The ncu summaries under profiles/ stay reproducible: each names the command
that made it, every ncu invocation keeps the GPU clocks unlocked
(--clock-control none), and the profiled program is a committed entry point
(bench.py or the q3b200 benchmark twin), never a scratch script."""
import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parents[1]
PROFILES = sorted((ROOT / "profiles").glob("*.md"))


def _commands(text: str) -> list[str]:
    blocks = re.findall(r"```\n(.*?)```", text, flags=re.S)
    return [b.replace("\\\n", " ") for b in blocks]


def test_every_summary_names_its_ncu_command():
    assert PROFILES
    for p in PROFILES:
        cmds = _commands(p.read_text())
        assert any("ncu " in c for c in cmds), p.name


def test_ncu_commands_leave_clocks_alone_and_run_committed_code():
    for p in PROFILES:
        text = p.read_text()
        assert "_work/" not in text, p.name
        for block in _commands(text):
            for line in block.splitlines():
                if "ncu " not in line or line.strip().startswith("#"):
                    continue
                assert "--clock-control none" in line, (p.name, line)
            targets = re.findall(r"python (?:-m (\S+)|(\S+\.py))", block)
            for mod, script in targets:
                if script:
                    assert (ROOT / script).exists(), (p.name, script)
                else:
                    assert mod.startswith("q3b200."), (p.name, mod)
                    path = ROOT / "qwen3-iree_b200" / (mod.replace(".", "/") + ".py")
                    assert path.exists(), (p.name, mod)
