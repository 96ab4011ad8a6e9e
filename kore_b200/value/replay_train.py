"""``kore value-train --inputs groups.jsonl --out value.json``."""
from __future__ import annotations

import argparse

from .model import train_from_groups


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore value-train")
    ap.add_argument("--inputs", required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    m = train_from_groups([p for p in a.inputs.split(",") if p])
    with open(a.out, "w") as f:
        f.write(m.to_json())
    print(f"[value-train] -> {a.out}")
    return 0
