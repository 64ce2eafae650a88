"""Extracts the known answers the reference's own tests and README state for
the projection path into reference_pins.json (committed beside this script).

The reference's numerical goldens, checkpoint and packs are not part of its
tree, so its tests can only pin counts, shapes, definitions and bars. This
script reads the reference sources as TEXT (nothing of it is built or run),
finds each pinned value by a pattern, and records the value together with the
file:line it came from. The tests read only the JSON.

    python tests/golden/make_reference_pins.py <reference root>
"""
from __future__ import annotations

import json
import re
import sys
from pathlib import Path


def find(root: Path, rel: str, pattern: str) -> tuple[int, re.Match]:
    lines = (root / rel).read_text(errors="replace").splitlines()
    rx = re.compile(pattern)
    for i, line in enumerate(lines, start=1):
        m = rx.search(line)
        if m:
            return i, m
    raise SystemExit(f"pattern {pattern!r} not found in {rel}")


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_reference_pins.py <reference root>")
    root = Path(sys.argv[1])
    pins = {}

    # quantized block matrices of a pack: CHECK(quant == 32 * 8 + 2 * 7)
    ln, m = find(root, "tests/ming-quant-test.cc",
                 r"CHECK\(quant == (\d+) \* (\d+) \+ (\d+) \* (\d+)\)")
    a, b, c, d = (int(g) for g in m.groups())
    pins["quantized_block_matrices"] = {
        "value": a * b + c * d, "modulated_blocks": a, "per_modulated_block": b,
        "refiner_blocks": c, "per_refiner_block": d,
        "source": f"tests/ming-quant-test.cc:{ln}"}
    ln, m = find(root, "tests/ming-quant-test.cc", r"CHECK\(dense_model == (\d+)\)")
    pins["dense_model_weights"] = {"value": int(m.group(1)),
                                   "source": f"tests/ming-quant-test.cc:{ln}"}
    # pack shape rule: codes [N, K*bits/32] beside scales [N, K/64]
    ln, m = find(root, "tests/ming-quant-test.cc",
                 r"ti->shape\[1\] \* (\d+) == si->shape\[1\] \* (\d+) \* bits")
    pins["pack_shape_rule"] = {"codes_word_bits": int(m.group(1)), "group": int(m.group(2)),
                               "source": f"tests/ming-quant-test.cc:{ln}"}
    # LoRA module capacity: 7 x (2 x refiner layers + layers); the real model's 238
    ln, m = find(root, "tests/ming-dit-test.cc",
                 r"want_mods == (\d+) \* \((\d+) \* d\.n_refiner_layers \+ d\.n_layers\)")
    pins["lora_capacity_rule"] = {"per_block": int(m.group(1)), "refiner_stacks": int(m.group(2)),
                                  "source": f"tests/ming-dit-test.cc:{ln}"}
    ln, m = find(root, "tests/ming-dit-test.cc", r"CHECK\(want == (\d+)\);")
    pins["lora_capacity_real_model"] = {"value": int(m.group(1)),
                                        "source": f"tests/ming-dit-test.cc:{ln}"}
    ln, m = find(root, "tests/ming-dit-test.cc", r"CHECK\(moved > ([0-9.]+)\);")
    pins["lora_moves_output_min_rel_l2"] = {"value": float(m.group(1)),
                                            "source": f"tests/ming-dit-test.cc:{ln}"}
    # relative L2 definition: sqrt(sum (a-b)^2 / sum b^2)
    ln, m = find(root, "tests/ming-test.h", r"return den > 0\.0 \? std::sqrt\(num / den\)")
    pins["rel_l2_definition"] = {"formula": "sqrt(sum((a-b)^2) / sum(b^2)), sqrt(num) if den == 0",
                                 "source": f"tests/ming-test.h:{ln}"}
    # bf16 forward vs fp32 forward bar stated by the README
    ln, m = find(root, "README.md", r"the reference's bf16: ([0-9.]+)")
    pins["bf16_forward_rel_l2_bar"] = {"value": float(m.group(1)), "source": f"README.md:{ln}"}

    out = Path(__file__).resolve().parent / "reference_pins.json"
    out.write_text(json.dumps(pins, indent=1, sort_keys=True) + "\n")
    print(f"wrote {out} ({len(pins)} pins)")


if __name__ == "__main__":
    main()
