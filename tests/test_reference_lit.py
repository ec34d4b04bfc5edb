"""The reference's own runtime tests (runtime/test/*.test, *.mlir), run against
this build's tools the way LLVM lit would run them.

The reference drives these files with lit and FileCheck, neither of which is
installed here, so this module is a small stand-in for both:
  - every `RUN:` line is run under bash with pipefail, after lit's
    substitutions: %hexir-run -> hexir-run, %hexir -> hexir-mkhxb (the
    stand-in for `hexir -emit=hxb`), %s / %S / %t -> the test file, its
    directory and a temporary path;
  - `not` inverts a command's status;
  - `FileCheck <file> [--check-prefix=P]` checks stdin against the file's
    P: / P-NEXT: lines, in order, with horizontal whitespace canonicalised
    (FileCheck's default).
The features lit would gate on are `runtime` and `compiler` (both present
here) and `cuda`, which this runner grants only when a CUDA GPU is visible;
a RUN line that needs one (`--device=cuda`) is skipped without a GPU.

The test files are read in place from the reference tree where it is
present (HEXIR_REFERENCE, else the checkout oracle/_ref was compiled from).
Without the tree -- on a GPU machine, where the files that require cuda
matter most -- the four .mlir files are rebuilt from tests/golden/
lit_cases.json (their RUN lines, check directives and programs, extracted
by tests/golden/make_golden.py --lit and pinned to the tree below); the two
.test files, which need the reference's fixture directory, then skip.
"""

import os
import re
import stat
import subprocess
import sys

import json

import pytest

from oracle import oracle
from tests.conftest import bin_path

LIT_CASES = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                         "lit_cases.json")


def ref_tests_dir():
    root = oracle.reference_root()
    return os.path.join(root, "runtime", "test") if root else None


FILES = ["fixture-cpu.test", "builtin-program.test", "hxb-roundtrip.mlir",
         "hxb-errors.mlir", "hxb-cuda.mlir", "hxb-cpu-vs-gpu.mlir"]

FILECHECK = r'''#!/usr/bin/env python3
import re, sys
args = sys.argv[1:]
prefix = "CHECK"
paths = []
for a in args:
    if a.startswith("--check-prefix="):
        prefix = a.split("=", 1)[1]
    else:
        paths.append(a)
def canon(s):
    return re.sub(r"[ \t]+", " ", s)
directive = re.compile(r"(?<![A-Za-z0-9_-])" + re.escape(prefix) + r"(-NEXT)?:(.*)$")
checks = []
for line in open(paths[0], encoding="utf-8", errors="replace"):
    m = directive.search(line.rstrip("\n"))
    if m:
        checks.append((bool(m.group(1)), canon(m.group(2).strip())))
if not checks:
    sys.exit("FileCheck: no %s: lines" % prefix)
text = [canon(l) for l in sys.stdin.read().split("\n")]
row, col = 0, 0
for nxt, pat in checks:
    if nxt:
        target = row + 1
        if target >= len(text) or pat not in text[target]:
            sys.exit("FileCheck: %s-NEXT: %r not on the line after %r"
                     % (prefix, pat, text[row] if row < len(text) else ""))
        row, col = target, text[target].index(pat) + len(pat)
        continue
    found = False
    r, c = row, col
    while r < len(text):
        i = text[r].find(pat, c)
        if i >= 0:
            row, col, found = r, i + len(pat), True
            break
        r, c = r + 1, 0
    if not found:
        sys.exit("FileCheck: %s: %r not found" % (prefix, pat))
'''

NOT = '''#!/bin/bash
"$@"
status=$?
if [ $status -eq 0 ]; then exit 1; fi
if [ $status -gt 128 ]; then exit $status; fi
exit 0
'''


def have_gpu() -> bool:
    try:
        import hexir_b200 as hx
        return hx.device_count() > 0
    except Exception:
        return False


def tools_dir(tmp_path):
    d = tmp_path / "bin"
    d.mkdir()
    for name, body in (("FileCheck", FILECHECK.replace(
            "#!/usr/bin/env python3", "#!" + sys.executable)), ("not", NOT)):
        p = d / name
        p.write_text(body)
        p.chmod(p.stat().st_mode | stat.S_IEXEC)
    return d


def run_lines(path):
    lines, current = [], ""
    for raw in open(path, encoding="utf-8"):
        m = re.search(r"RUN:(.*)$", raw.rstrip("\n"))
        if not m:
            continue
        part = m.group(1).strip()
        if part.endswith("\\"):
            current += part[:-1] + " "
            continue
        lines.append(current + part)
        current = ""
    return lines


def requires(path):
    feats = set()
    for raw in open(path, encoding="utf-8"):
        m = re.search(r"REQUIRES:(.*)$", raw)
        if m:
            feats |= {f.strip() for f in m.group(1).split(",") if f.strip()}
    return feats


def fixture_cases():
    with open(LIT_CASES) as f:
        return {os.path.basename(c["file"]): c for c in json.load(f)["cases"]}


def materialize(cases, dest):
    """Write each fixture case back as a lit file: its program, then its
    REQUIRES, RUN and check lines as comments."""
    for name, case in cases.items():
        lines = list(case["program"]) + [""]
        if case["requires"]:
            lines.append("// REQUIRES: " + ", ".join(case["requires"]))
        lines += ["// RUN: " + r for r in case["run"]]
        for prefix, checks in case["checks"].items():
            lines += [f"// {prefix}{'-NEXT' if nxt else ''}: {pat}"
                      for nxt, pat in checks]
        (dest / name).write_text("\n".join(lines) + "\n")


def lit_path(tmp_path, name):
    """The lit file `name`: in place in the reference tree, else rebuilt
    from the fixture; None when neither has it."""
    tree = ref_tests_dir()
    if tree and os.path.exists(os.path.join(tree, name)):
        return os.path.join(tree, name)
    cases = fixture_cases()
    if name not in cases:
        return None
    d = tmp_path / "lit"
    d.mkdir()
    materialize(cases, d)
    return str(d / name)


def test_lit_fixture_matches_the_reference_tree():
    tree = ref_tests_dir()
    if not tree:
        pytest.skip("the reference tree is not present here")
    sys.path.insert(0, os.path.dirname(LIT_CASES))
    import make_golden
    for name, case in fixture_cases().items():
        assert make_golden.lit_case(os.path.join(tree, name)) == case, name


def test_rebuilt_lit_file_reads_back_the_same(tmp_path):
    """The rebuilt files give the runner the same RUN lines and checks."""
    sys.path.insert(0, os.path.dirname(LIT_CASES))
    import make_golden
    cases = fixture_cases()
    materialize(cases, tmp_path)
    for name, case in cases.items():
        got = make_golden.lit_case(str(tmp_path / name))
        assert {k: v for k, v in got.items() if k != "file"} == \
            {k: v for k, v in case.items() if k != "file"}, name


def run_lit_file(tmp_path, path, gpu):
    """Every RUN line of one lit file; returns (ran, skipped) lines."""
    env = dict(os.environ,
               PATH=str(tools_dir(tmp_path)) + os.pathsep + os.environ["PATH"])
    ran, skipped = 0, []
    for line in run_lines(path):
        if "--device=cuda" in line and not gpu:
            skipped.append(line)
            continue
        cmd = (line.replace("%hexir-run", bin_path("hexir-run"))
                   .replace("%hexir", bin_path("hexir-mkhxb"))
                   .replace("%s", path)
                   .replace("%S", os.path.dirname(path))
                   .replace("%t", str(tmp_path / "t")))
        res = subprocess.run(["bash", "-o", "pipefail", "-c", cmd], env=env,
                             capture_output=True, text=True, timeout=300)
        assert res.returncode == 0, (
            f"{os.path.basename(path)}: RUN: {line}\n--- stdout\n{res.stdout}"
            f"\n--- stderr\n{res.stderr}")
        ran += 1
    return ran, skipped


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["hxb-cuda.mlir", "hxb-cpu-vs-gpu.mlir",
                                  "hxb-errors.mlir"])
def test_reference_cuda_lit_files_on_the_gpu(tmp_path, name):
    """On a GPU machine (where the reference tree is absent, so the files
    come from the fixture): every RUN line, the `--device=cuda` ones
    included -- the CPU-vs-GPU diff, the GPU known answer, the misplaced
    module refused on a CPU device, the CUDA HAL self-test."""
    assert have_gpu(), "gpu-marked tests run where a GPU is expected"
    path = lit_path(tmp_path, name)
    assert path is not None
    ran, skipped = run_lit_file(tmp_path, path, gpu=True)
    assert ran == len(run_lines(path)) and not skipped


@pytest.mark.parametrize("name", FILES)
def test_reference_runtime_lit_file(tmp_path, name):
    path = lit_path(tmp_path, name)
    if path is None:
        pytest.skip("needs the reference tree (its fixture directory)")
    gpu = have_gpu()
    missing = requires(path) - {"runtime", "compiler"} - ({"cuda"} if gpu else set())
    if missing:
        pytest.skip(f"needs {sorted(missing)} (lit would mark it UNSUPPORTED)")
    ran, skipped = run_lit_file(tmp_path, path, gpu)
    assert ran > 0
    # Only the CUDA HAL self-test of hxb-errors.mlir needs a GPU outside the
    # files that require cuda.
    assert len(skipped) <= 1, skipped


def test_filecheck_stand_in_rejects_what_filecheck_rejects(tmp_path):
    """The stand-in fails on a missing line, a CHECK-NEXT that is not on the
    next line, and out-of-order lines, and passes the same input otherwise;
    `not` inverts a status."""
    d = tools_dir(tmp_path)
    checks = tmp_path / "c.txt"
    checks.write_text("# CHECK: alpha   1\n# CHECK-NEXT: beta\n# CHECK: gamma\n"
                      "# X: only-x\n")
    def fc(text, *extra):
        return subprocess.run([str(d / "FileCheck"), str(checks), *extra],
                              input=text, capture_output=True, text=True).returncode
    assert fc("pre\nalpha 1\nbeta\nmid\ngamma\n") == 0
    assert fc("alpha\t 1 x\nbeta 2\ngamma") == 0        # whitespace canonicalised
    assert fc("alpha 1\nmid\nbeta\ngamma\n") != 0        # NEXT not next
    assert fc("gamma\nalpha 1\nbeta\n") != 0             # order
    assert fc("alpha 1\nbeta\n") != 0                    # missing
    assert fc("only-x\n", "--check-prefix=X") == 0
    assert fc("nothing\n", "--check-prefix=X") != 0
    assert subprocess.run([str(d / "not"), "false"]).returncode == 0
    assert subprocess.run([str(d / "not"), "true"]).returncode != 0
