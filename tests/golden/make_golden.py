#!/usr/bin/env python3
"""Generate tests/golden/golden.json from the reference implementation itself.

Run in a container that has the reference tree and the reference runtime
built from its own sources (`make -C oracle ref`):

    python tests/golden/make_golden.py [--reference <reference checkout>]

It records (golden.json)
  - the reference's checked-in CPU fixture (runtime/test/fixtures/mlp-cpu.hxb):
    size, sha256 and what the reference hexir-run prints for it;
  - known-answer programs from the reference's runtime tests, written here as
    our own programs with the same matrices, and the reference hexir-run's
    stdout for each (run on modules produced by this project's writer,
    placement all cpu);
  - seeded matmul / relu / add vectors: inputs from the writer's SplitMix64
    stream (small shapes and the 256x256 seed-0 parity graph), outputs of the
    reference's own hexir_ref_*_f64 kernels, stored as sha256 of the output
    bytes plus a few sampled values.

With --lit it writes lit_cases.json instead: for each of the reference's
runtime lit tests that need no fixture files (runtime/test/*.mlir), its
REQUIRES features, RUN lines, check directives and program, so that
tests/test_reference_lit.py runs them where the reference tree is absent
(a GPU machine, for the files that require cuda).

The tests then need neither the reference tree nor the reference library,
so they also run on machines that have neither.
"""

import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import hexir_b200 as hx  # noqa: E402
from oracle import oracle  # noqa: E402

# Programs with the matrices of the reference's runtime tests.
KNOWN_ANSWERS = [
    {  # runtime/test/hxb-cuda.mlir:19-30, fixture-cpu.test:19-21
        "name": "linear_2x2",
        "source": "runtime/test/hxb-cuda.mlir",
        "a": [[3.0, 1.0], [2.0, 2.0]], "b": [[1.0, 5.0], [5.0, 2.0]],
        "ops": ["linear"],
    },
    {  # runtime/test/hxb-roundtrip.mlir:10-30
        "name": "linear_add_relu_2x2",
        "source": "runtime/test/hxb-roundtrip.mlir",
        "a": [[3.0, 1.0], [2.0, 2.0]], "b": [[1.0, 5.0], [5.0, 2.0]],
        "ops": ["linear", "add_b", "relu"],
    },
    {  # runtime/test/hxb-cpu-vs-gpu.mlir:18-29
        "name": "linear_relu_negatives_2x2",
        "source": "runtime/test/hxb-cpu-vs-gpu.mlir",
        "a": [[3.0, -1.0], [2.0, 2.0]], "b": [[1.0, 5.0], [5.0, -2.0]],
        "ops": ["linear", "relu"],
    },
]

MATMUL_VECTORS = [
    (1, 1, 1, 10), (2, 3, 4, 11), (37, 53, 29, 12), (64, 64, 64, 13),
    (100, 7, 300, 14), (5, 129, 67, 15), (256, 256, 256, 0),
]


def build_known(case):
    p = hx.Program()
    a = p.constant(np.array(case["a"]))
    b = p.constant(np.array(case["b"]))
    v = p.linear(a, b)
    for op in case["ops"][1:]:
        if op == "add_b":
            v = p.add(v, b)
        elif op == "relu":
            v = p.relu(v)
    p.print(v)
    return p


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def seeded_inputs(m, n, k, seed):
    rng = hx.Rng(seed)
    return rng.uniform((m, k)), rng.uniform((k, n))


LIT_FILES = ["hxb-roundtrip.mlir", "hxb-errors.mlir", "hxb-cuda.mlir",
             "hxb-cpu-vs-gpu.mlir"]


def lit_case(path: str) -> dict:
    """What a lit run of one reference runtime test needs, read from the
    file: its REQUIRES features, its RUN lines (continuations joined), its
    check directives by prefix, and the program (the lines that are not
    comments)."""
    import re
    requires, run, checks, program = [], [], {}, []
    current = ""
    directive = re.compile(r"^//\s*([A-Z][A-Z0-9_]*)(-NEXT)?:(.*)$")
    for raw in open(path, encoding="utf-8"):
        line = raw.rstrip("\n")
        m = re.search(r"REQUIRES:(.*)$", line)
        if m:
            requires += [f.strip() for f in m.group(1).split(",") if f.strip()]
            continue
        m = re.search(r"RUN:(.*)$", line)
        if m:
            part = m.group(1).strip()
            if part.endswith("\\"):
                current += part[:-1] + " "
            else:
                run.append(current + part)
                current = ""
            continue
        m = directive.match(line.strip())
        if m and m.group(1) not in ("REQUIRES", "RUN"):
            checks.setdefault(m.group(1), []).append(
                [bool(m.group(2)), m.group(3).strip()])
            continue
        if not line.lstrip().startswith("//"):
            program.append(line)
    while program and not program[0].strip():
        program.pop(0)
    while program and not program[-1].strip():
        program.pop()
    return {"file": "runtime/test/" + os.path.basename(path),
            "requires": requires, "run": run, "checks": checks,
            "program": program}


def write_lit_cases(reference: str) -> None:
    cases = [lit_case(os.path.join(reference, "runtime/test", name))
             for name in LIT_FILES]
    dest = os.path.join(HERE, "lit_cases.json")
    with open(dest, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py --lit",
                   "cases": cases}, f, indent=1)
    print("wrote", dest)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=oracle.reference_root(),
                    help="the reference checkout (default: HEXIR_REFERENCE, "
                         "else the one oracle/_ref was built from)")
    ap.add_argument("--lit", action="store_true",
                    help="only write lit_cases.json: the reference runtime "
                         "tests' RUN lines, checks and programs")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("set HEXIR_REFERENCE or pass --reference")
    if args.lit:
        write_lit_cases(args.reference)
        return
    if not oracle.have_reference():
        raise SystemExit("build the reference runtime first: make -C oracle ref")
    ref_run = oracle.REF_RUN
    out = {"generator": "tests/golden/make_golden.py",
           "reference_runtime": "oracle/_ref (reference runtime/ sources, gcc -O2)"}

    fixture = os.path.join(args.reference, "runtime/test/fixtures/mlp-cpu.hxb")
    blob = open(fixture, "rb").read()
    stdout = subprocess.run([ref_run, "--quiet", fixture], capture_output=True,
                            text=True, check=True).stdout
    out["reference_fixture"] = {
        "path": "runtime/test/fixtures/mlp-cpu.hxb", "size": len(blob),
        "sha256": hashlib.sha256(blob).hexdigest(), "stdout_quiet": stdout}

    known = []
    with tempfile.TemporaryDirectory() as tmp:
        for case in KNOWN_ANSWERS:
            path = os.path.join(tmp, case["name"] + ".hxb")
            build_known(case).emit_file(path)
            res = subprocess.run([ref_run, "--quiet", path], capture_output=True,
                                 text=True, check=True)
            known.append({**case, "stdout_quiet": res.stdout})
    out["known_answers"] = known

    vectors = []
    for m, n, k, seed in MATMUL_VECTORS:
        a, b = seeded_inputs(m, n, k, seed)
        c = oracle.ref_matmul(a, b)
        r = oracle.ref_relu(c)
        s = oracle.ref_add(c, c[::-1].copy())
        vectors.append({
            "m": m, "n": n, "k": k, "seed": seed,
            "inputs": "writer SplitMix64 uniform[-1,1): a [m x k] then b [k x n]",
            "matmul_sha256": sha(c), "relu_sha256": sha(r),
            "add_reversed_rows_sha256": sha(s),
            "samples": [[int(i), int(j), float(c[i, j])]
                        for i, j in [(0, 0), (m - 1, n - 1), (m // 2, n // 3)]],
        })
    out["matmul_vectors"] = vectors

    special = np.array([0.0, -0.0, 1.5, -1.5, np.inf, -np.inf, np.nan,
                        5e-324, -5e-324, 1e308, -1e308])
    out["relu_specials"] = {
        "input_hex": [float(x).hex() for x in special],
        "output_bits": [int(v) for v in oracle.ref_relu(special).view(np.uint64)],
    }

    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "golden.json"))


if __name__ == "__main__":
    main()
