#!/usr/bin/env python3
"""Regenerate the golden fixtures from the reference project's own oracle.

Runs only where the reference checkout is mounted (the build container);
the committed outputs travel, this script's inputs do not.  It imports the
reference's CPU oracle ``operator/tests/triangle_v2_reference.py`` read-only
and reads the parameters of the reference's NPU correctness matrix
(``operator/tests/npu_v2_correctness.py:51-216``, ``DEFAULT_CASES``, 18 cases) with
``ast`` (that module itself imports torch_npu and cannot be imported here).

Outputs (next to this script):
  reference_cases.json  case parameters, sha256 of the generated inputs,
                        stored row indices, sentinel values
  reference_cases.npz   reference outputs (float32) of the stored rows
  intervals.json        reference ``selected_intervals`` over a grid of rows

Usage:  python tests/golden/make_golden.py --reference <reference checkout>
"""

from __future__ import annotations

import argparse
import ast
import importlib.util
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from inputs import SCALE, inputs_digest, reference_case_inputs  # noqa: E402


def load_reference(ref_root: Path):
    path = ref_root / "operator/tests/triangle_v2_reference.py"
    spec = importlib.util.spec_from_file_location("triangle_v2_reference", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["triangle_v2_reference"] = mod
    spec.loader.exec_module(mod)
    return mod


def read_cases(ref_root: Path) -> list[dict]:
    src = (ref_root / "operator/tests/npu_v2_correctness.py").read_text()
    tree = ast.parse(src)
    cases = []
    for node in ast.walk(tree):
        if isinstance(node, ast.Call) and getattr(node.func, "id", "") == "CorrectnessCase":
            vals = [ast.literal_eval(a) for a in node.args]
            name, q0, tq, seq, prompt, seed, coverage = vals
            cases.append(dict(name=name, query_start=q0, query_tokens=tq, seq_len=seq,
                              prompt_len=prompt, seed=seed, coverage=coverage))
    if len(cases) < 17:
        raise RuntimeError(f"expected the reference's correctness cases, found {len(cases)}")
    return cases


def pick_rows(case: dict) -> list[int]:
    tq, q0, prompt = case["query_tokens"], case["query_start"], case["prompt_len"]
    if tq <= 4:
        return list(range(tq))
    boundary = {0, tq - 1}
    for absolute in (520, 521, prompt - 129, prompt - 128):
        if q0 <= absolute < q0 + tq:
            boundary.add(absolute - q0)
    rows = sorted(boundary)
    extra = [r for r in (tq // 3, (2 * tq) // 3) if r not in boundary]
    return sorted(set(rows + extra))[:6]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True,
                    help="root of the reference project checkout")
    args = ap.parse_args()
    ref = load_reference(args.reference)
    torch.set_num_threads(8)

    meta = {"scale": SCALE, "cases": [], "sentinels": {}}
    arrays = {}
    for case in read_cases(args.reference):
        q, k, v, table = reference_case_inputs(case["query_start"], case["query_tokens"],
                                               case["seq_len"], case["seed"])
        out = ref.torch_reference_attention(q, k, v, table, case["query_start"], case["seq_len"],
                                            case["prompt_len"], SCALE)
        rows = pick_rows(case)
        arrays[case["name"]] = out[rows].numpy().astype(np.float32)
        meta["cases"].append({**case, "rows": rows, "digest": inputs_digest(q, k, v, table),
                              "table": table[0].tolist()})
        print(f"{case['name']}: rows {rows}")

    # Shared-softmax sentinel (reference npu_v2_correctness.py:401-473).
    gen = torch.Generator().manual_seed(2201)
    logical = math.ceil(522 / 128)
    perm = torch.randperm(logical + 5, generator=gen, dtype=torch.int64)[:logical]
    table = perm.to(torch.int32).view(1, -1)
    shape = (logical + 5, 128, 8, 128)
    kz = torch.zeros(shape, dtype=torch.bfloat16)
    vz = torch.zeros(shape, dtype=torch.bfloat16)

    def put(tokens, value):
        for t in tokens:
            p, o = ref.physical_location(t, table[0].tolist(), ref.PRODUCTION_GEOMETRY)
            vz[p, o].fill_(value)

    put(range(8), 10.0)
    put((8,), 1000.0)
    put(range(9, 522), 1.0)
    qz = torch.zeros(1, 32, 128, dtype=torch.bfloat16)
    out = ref.torch_reference_attention(qz, kz, vz, table, 521, 522, 2048, SCALE)
    meta["sentinels"]["shared_softmax"] = {
        "table": table[0].tolist(), "pages": logical + 5, "value": float(out[0, 0, 0]),
        "joint_expected": (8.0 * 10.0 + 513.0) / 521.0, "forbidden": 11.0}

    # Interval grid from the reference schedule.
    grid = []
    for prompt in (600, 649, 650, 1024, 2048, 8192, 8320):
        for seq in sorted({min(prompt, s) for s in (1, 255, 521, 522, 600, 1024, prompt)}):
            for qpos in sorted({0, 7, 8, 9, 519, 520, 521, 522, 895, 896, seq - 129, seq - 128,
                                seq - 1, prompt - 129, prompt - 128}):
                if 0 <= qpos < seq:
                    grid.append([qpos, seq, prompt,
                                 [list(iv) for iv in ref.selected_intervals(qpos, seq, prompt)]])
    (HERE / "intervals.json").write_text(json.dumps(grid, separators=(",", ":")) + "\n")
    (HERE / "reference_cases.json").write_text(json.dumps(meta, indent=1) + "\n")
    np.savez_compressed(HERE / "reference_cases.npz", **arrays)
    print("wrote", len(meta["cases"]), "cases,", len(grid), "interval rows")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
