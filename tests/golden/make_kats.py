"""Extract the optimizer-path known-answer values from the reference's own tests.

The reference (dhilipsiva/python-slm) is Rust and cannot be built here, so its
golden vectors are read out of its test sources as text and written to
reference_kats.json next to this script.  Each value records the file:line it
came from.  Run once where the reference tree is mounted, giving its root:

    python tests/golden/make_kats.py <path to the python-slm checkout>

The tests only read the committed JSON; nothing at test time touches the
reference tree.
"""
from __future__ import annotations

import json
import re
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "reference_kats.json"


def find(root: Path, rel: str, pattern: str, flags=0):
    text = (root / rel).read_text()
    m = re.search(pattern, text, flags)
    if not m:
        raise SystemExit(f"pattern not found in {rel}: {pattern}")
    line = text[: m.start()].count("\n") + 1
    return m, f"{rel}:{line}"


def num(s: str) -> int:
    return int(s.replace("_", ""), 0)


def main(root: Path) -> None:
    kats: dict = {"source": "dhilipsiva/python-slm test sources", "values": {}}
    v = kats["values"]

    # bf16 round-to-nearest-even, src/model/oracle.rs tests
    m, at = find(root, "src/model/oracle.rs",
                 r"f32_to_bf16_bits\(1\.0\), (0x[0-9a-f]+)\);")
    cases = [{"f32_bits": "0x3f800000", "bf16": m.group(1), "at": at}]
    for mm in re.finditer(r"f32_to_bf16_bits\(f32::from_bits\((0x[0-9a-f_]+)\)\), (0x[0-9a-f]+)\);",
                          (root / "src/model/oracle.rs").read_text()):
        text = (root / "src/model/oracle.rs").read_text()
        line = text[: mm.start()].count("\n") + 1
        cases.append({"f32_bits": hex(num(mm.group(1))), "bf16": mm.group(2),
                      "at": f"src/model/oracle.rs:{line}"})
    v["bf16_rne"] = cases

    # gradient_clip_scale and adamw_scalar_step
    m, at = find(root, "src/model/oracle.rs",
                 r"gradient_clip_scale\(&\[3\.0, 4\.0\]\)\.unwrap\(\)\.to_bits\(\),\s*([0-9.]+)_f32\.to_bits\(\)")
    v["clip_3_4"] = {"input": [3.0, 4.0], "expected_f32": float(m.group(1)), "at": at}
    m, at = find(root, "src/model/oracle.rs",
                 r"gradient_clip_scale\(&\[0\.0, 0\.0\]\)\.unwrap\(\), ([0-9.]+)\)")
    v["clip_zero"] = {"input": [0.0, 0.0], "expected_f32": float(m.group(1)), "at": at}
    m, at = find(root, "src/model/oracle.rs",
                 r"gradient_clip_scale\(&\[f32::NAN\]\)\.unwrap_err\(\)\.code,\s*\"([A-Z_]+)\"")
    v["clip_nan"] = {"expected_code": m.group(1), "at": at}
    m, at = find(root, "src/model/oracle.rs",
                 r"adamw_scalar_step\(([0-9.]+), ([0-9.]+), ([0-9.]+), ([0-9.]+), ([0-9.]+), (\d+), ([0-9.]+)\)\.unwrap\(\);\s*"
                 r"assert_eq!\(moment\.to_bits\(\), ([0-9_]+)\);\s*assert_eq!\(variance\.to_bits\(\), ([0-9_]+)\);")
    v["adamw_step"] = {
        "theta": float(m.group(1)), "gradient": float(m.group(2)), "moment": float(m.group(3)),
        "variance": float(m.group(4)), "learning_rate": float(m.group(5)), "t": int(m.group(6)),
        "weight_decay": float(m.group(7)), "moment_bits": num(m.group(8)),
        "variance_bits": num(m.group(9)), "master_below": 1.0, "storage_is_rne_of_master": True,
        "at": at}

    # optimizer rules, tests/p9b_model_oracle.rs
    rules = {}
    for key in ("beta1", "beta2", "epsilon", "decay_weight", "no_decay_weight", "global_l2_clip"):
        m, at = find(root, "tests/p9b_model_oracle.rs",
                     rf"rules\.{key}\.to_bits\(\), ([0-9.e\-]+)_f32\.to_bits\(\)")
        rules[key] = {"value_f32": float(m.group(1)), "at": at}
    m, at = find(root, "tests/p9b_model_oracle.rs", r'rules\.algorithm, "([a-z0-9\-]+)"')
    rules["algorithm"] = {"value": m.group(1), "at": at}
    v["optimizer_rules"] = rules

    # layout: tensor count, parameter count, layout SHA, decay groups
    m, at = find(root, "tests/p9b_model_oracle.rs",
                 r'parameter_layout_sha256\(&specs\),\s*"([0-9a-f]{64})"')
    v["layout_sha256"] = {"value": m.group(1), "at": at}
    m, at = find(root, "src/model.rs", r"CANONICAL_PARAMETER_COUNT: u64 = ([0-9_]+);")
    v["canonical_parameter_count"] = {"value": num(m.group(1)), "at": at}
    m, at = find(root, "src/model.rs", r"REFERENCE_PARAMETER_COUNT: u64 = ([0-9_]+);")
    v["reference_parameter_count"] = {"value": num(m.group(1)), "at": at}
    m, at = find(root, "src/model/oracle.rs", r"assert_eq!\(specs\.len\(\), (\d+)\);")
    v["tensor_count"] = {"value": int(m.group(1)), "at": at}
    m, at = find(root, "src/model/oracle.rs",
                 r"OptimizerGroup::NoDecay\)\s*\.count\(\),\s*(\d+)\s*\);")
    v["no_decay_tensor_count"] = {"value": int(m.group(1)), "at": at}
    names = {}
    for mm in re.finditer(r'assert_eq!\(specs\[(\d+)\]\.name, "([a-z0-9_.]+)"\);',
                          (root / "src/model/oracle.rs").read_text()):
        names[mm.group(1)] = mm.group(2)
    v["tensor_names"] = {"value": names, "at": "src/model/oracle.rs:1352-1361"}
    shapes = {}
    for mm in re.finditer(r"assert_eq!\(specs\[(\d+)\]\.shape, \[([0-9_, ]+)\]\);",
                          (root / "src/model/oracle.rs").read_text()):
        shapes[mm.group(1)] = [num(x.strip()) for x in mm.group(2).split(",")]
    v["tensor_shapes"] = {"value": shapes, "at": "src/model/oracle.rs:1353-1357"}

    # trainer constants
    consts = {}
    for key in ("TARGETS_PER_FULL_UPDATE", "FINAL_UPDATE_TARGETS", "TOTAL_UPDATES",
                "WARMUP_UPDATES"):
        m, at = find(root, "src/train/trainer.rs", rf"pub const {key}: u64 = ([0-9_]+);")
        consts[key] = {"value": num(m.group(1)), "at": at}
    for key in ("PEAK_LEARNING_RATE", "MINIMUM_LEARNING_RATE", "CLIP_VERIFICATION_TOLERANCE"):
        m, at = find(root, "src/train/trainer.rs", rf"pub const {key}: f32 = ([0-9.e\-]+);")
        consts[key] = {"value_f32": float(m.group(1)), "at": at}
    v["trainer_constants"] = consts

    # p12 production-width clip probe
    m, at = find(root, "tests/p12_trainer.rs",
                 r"for count in \[\s*([0-9_]+)_usize,\s*([0-9_]+),\s*([0-9_]+),\s*CANONICAL_PARAMETER_COUNT")
    m2, at2 = find(root, "tests/p12_trainer.rs",
                   r"\(\(index % (\d+)\) as f32 - ([0-9.]+)\) \* ([0-9.e\-]+)")
    v["clip_probe"] = {"counts": [num(m.group(i)) for i in (1, 2, 3)] + ["CANONICAL"],
                       "modulus": int(m2.group(1)), "offset": float(m2.group(2)),
                       "scale": float(m2.group(3)), "at": [at, at2]}

    # e1 codec round trip gradients
    m, at = find(root, "tests/e1_full_model_backend.rs",
                 r"if index % (\d+) == 0 \{ ([0-9.\-]+) \} else \{ ([0-9.\-]+) \}")
    m2, at2 = find(root, "tests/e1_full_model_backend.rs", r"assert_eq!\(elements, (\d+)\);")
    v["e1_codec"] = {"modulus": int(m.group(1)), "hit": float(m.group(2)),
                     "miss": float(m.group(3)), "elements": int(m2.group(1)), "at": [at, at2]}

    OUT.write_text(json.dumps(kats, indent=1, sort_keys=True) + "\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_kats.py <path to the python-slm checkout>")
    main(Path(sys.argv[1]))
