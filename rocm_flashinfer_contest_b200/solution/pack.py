"""Packs the B200 GDN solutions into flashinfer-bench solution.json files.

The JSON layout is the harness's Solution schema, the same fields the
reference's tools/pack_solution.py:33-46 writes: name, definition, author,
spec {language, target_hardware, entry_point, dependencies,
destination_passing_style}, sources [{path, content}], description.  Each
solution embeds one main.py whose `run` is this package's entry point.

    python -m rocm_flashinfer_contest_b200.solution.pack --out-dir solutions_b200
"""
from __future__ import annotations

import argparse
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))

# (definition, solution name, main.py source file)
SOLUTIONS = [
    ("gdn_decode_qk4_v8_d128_k_last", "gdn_decode_b200_v1", "gdn_decode_main.py"),
    ("gdn_prefill_qk4_v8_d128_k_last", "gdn_prefill_b200_v1", "gdn_prefill_main.py"),
]


def solution_dict(definition: str, name: str, main_file: str) -> dict:
    with open(os.path.join(HERE, main_file)) as f:
        content = f.read()
    return {
        "name": name,
        "definition": definition,
        "author": "b200-gdn",
        "spec": {
            "language": "python",
            "target_hardware": ["NVIDIA B200"],
            "entry_point": "main.py::run",
            "dependencies": ["torch", "rocm_flashinfer_contest_b200"],
            "destination_passing_style": False,
        },
        "sources": [{"path": "main.py", "content": content}],
        "description": f"B200 sm_100a CUDA kernels (tcgen05 prefill, HBM-streaming decode) for {definition}",
    }


def pack(out_dir: str) -> list[str]:
    os.makedirs(out_dir, exist_ok=True)
    paths = []
    for definition, name, main_file in SOLUTIONS:
        path = os.path.join(out_dir, definition.split("_qk")[0], "solution.json")
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as f:
            json.dump(solution_dict(definition, name, main_file), f, indent=2)
        paths.append(path)
    return paths


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out-dir", default="solutions_b200")
    args = ap.parse_args()
    for p in pack(args.out_dir):
        print("wrote", p)


if __name__ == "__main__":
    main()
