"""The README's commands and environment switches stay in step with the code.

Every `hetero_cp_ringattn_b200 <command> ...` and `bench.py ...` line in the README parses with
the real argument parsers, and every `HCP_*` switch the README names is read somewhere in the
package's sources; the README's Python example runs (on the CPU here).
"""

import pathlib
import re
import shlex

import pytest

from hetero_cp_ringattn_b200.cli import build_parser

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _readme_commands():
    """Shell lines of the README's code blocks, continuation lines joined, comments dropped."""
    lines, out, buf, fenced = ROOT.joinpath("README.md").read_text().splitlines(), [], "", None
    for ln in lines:
        if ln.startswith("```"):
            fenced = ln[3:].strip() if fenced is None else None
            continue
        if fenced != "" or ln.lstrip().startswith("#"):
            continue
        code = ln.split(" #", 1)[0].rstrip()
        if code.endswith("\\"):
            buf += code[:-1] + " "
            continue
        buf += code
        if buf.strip():
            out.append(buf.strip())
        buf = ""
    return out


def _after(cmd, marker):
    toks = shlex.split(cmd)
    return toks[toks.index(marker) + 1:]


CLI = [c for c in _readme_commands() if "hetero_cp_ringattn_b200" in shlex.split(c)]
BENCH = [c for c in _readme_commands() if "bench.py" in shlex.split(c)]


def test_readme_has_commands_to_check():
    assert len(CLI) >= 6 and len(BENCH) >= 3


@pytest.mark.parametrize("cmd", CLI)
def test_readme_cli_commands_parse(cmd):
    args = build_parser().parse_args(_after(cmd, "hetero_cp_ringattn_b200"))
    assert callable(args.fn)


@pytest.mark.parametrize("cmd", BENCH)
def test_readme_bench_commands_parse(cmd):
    import bench
    args = bench.parse(_after(cmd, "bench.py"))
    assert args.gpus >= 1 and args.warmup >= 3


def test_readme_environment_switches_are_read_by_the_code():
    readme = ROOT.joinpath("README.md").read_text()
    names = set(re.findall(r"\bHCP_[A-Z0-9_]+", readme))
    assert len(names) >= 8
    src = "\n".join(p.read_text(errors="replace")
                    for ext in ("*.py", "*.cu", "*.cuh", "*.h", "*.cpp")
                    for p in ROOT.joinpath("hetero_cp_ringattn_b200").rglob(ext))
    src += ROOT.joinpath("setup.py").read_text()
    missing = sorted(n for n in names if f'"{n}"' not in src)
    assert not missing, missing


def test_readme_python_example_runs():
    text = ROOT.joinpath("README.md").read_text()
    blocks = re.findall(r"```python\n(.*?)```", text, re.S)
    assert len(blocks) == 1
    scope = {}
    exec(compile(blocks[0], "README.md", "exec"), scope)
    ids, eng = scope["ids"], scope["eng"]
    assert ids.numel() == 8 and not eng.reqs
