"""``kore value-train --inputs groups.jsonl[,more.jsonl] --out value.json``

Fits the value model from ranked-group records (the datagen ``groups``
output). ``--synthetic N`` fits a cold-start model from N synthetic groups
with a known ground truth instead (``kore_b200.value.features.synthesize_groups``),
and ``--holdout`` reports the within-group Spearman correlation of the fitted
model on fresh synthetic groups. Reference parity: kore/value/replay_train.py:152
and train_value.py:54-443.
"""
from __future__ import annotations

import argparse
import json

from .model import ValueModel, train_from_groups


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore value-train")
    ap.add_argument("--inputs", default="")
    ap.add_argument("--out", required=True)
    ap.add_argument("--synthetic", type=int, default=0, help="fit from N synthetic groups instead")
    ap.add_argument("--holdout", type=int, default=0, help="synthetic held-out groups to report on")
    ap.add_argument("--featurizer", default="v2", choices=["v1", "v2"])
    a = ap.parse_args(argv)
    if a.synthetic:
        from .features import synthesize_groups
        m = ValueModel(a.featurizer).fit_groups(synthesize_groups(a.synthetic, seed=0))
    else:
        paths = [p for p in a.inputs.split(",") if p]
        if not paths:
            ap.error("--inputs or --synthetic is required")
        m = train_from_groups(paths, featurizer=a.featurizer)
    with open(a.out, "w") as f:
        f.write(m.to_json())
    report = {"out": a.out, "featurizer": m.featurizer}
    if a.holdout:
        from .features import synthesize_groups
        from .rerank import groupwise_spearman

        def score(rows):
            return list(m.predict(m.featurize([r["source"] for r in rows], rows[0].get("meta")))["utility"])
        report["holdout_spearman"] = groupwise_spearman(score, synthesize_groups(a.holdout, seed=12345))
    print(json.dumps(report))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
