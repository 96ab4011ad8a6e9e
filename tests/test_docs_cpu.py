"""Every source path named in the design notes' component table exists
(brace lists and globs expanded), so the map from blueprint to code cannot
go stale silently."""
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _expand(p: str):
    m = re.search(r"\{([^}]*)\}", p)
    if not m:
        return [p]
    out = []
    for alt in m.group(1).split(","):
        out += _expand(p[: m.start()] + alt.strip() + p[m.end():])
    return out


def test_design_table_paths_exist():
    text = open(os.path.join(ROOT, "DESIGN.md")).read()
    paths = set(re.findall(r"`((?:kore_b200|baseline|tests)/[^`\s]+)`", text))
    assert len(paths) > 40
    missing = []
    for p in paths:
        for q in _expand(p):
            q = q.rstrip("/")
            hits = glob.glob(os.path.join(ROOT, q))
            if not hits and not os.path.exists(os.path.join(ROOT, q)):
                missing.append(q)
    assert not missing, missing
