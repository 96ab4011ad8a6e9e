"""Mid-training (continued pretraining) corpus for the B200 domain.

The policy enters SFT fluent in the world it will write kernels for: CUDA on
sm_100a (tcgen05, TMEM, TMA, clusters), CUTLASS / CuTe, Triton on Blackwell,
PyTorch operator semantics. The corpus is assembled offline and
deterministically from sources on the machine:

* ``tasks``: every registered task's operator definition, fp32 oracle source
  and seed kernel, as one document per task (held-out tasks excluded);
* ``repo_kernels``: this repository's own sm_100a CUDA sources and their
  Python bindings (``kore_b200/csrc``, ``kore_b200/ops``);
* ``cutlass``: CUTLASS / CuTe header trees found in installed packages
  (sm100 collectives and atoms first);
* ``triton``: Triton kernel files of installed packages (files that define a
  ``@triton.jit`` function);
* ``docs``: Markdown / reStructuredText documentation next to those sources,
  and this repository's B200 playbook;
* ``wins``: final kernels of verified optimisation wins (when given).

Every file goes through the quality filters of
:mod:`kore_b200.data.corpus_quality`, long files are cut at line boundaries
into chunks of ``chunk_chars``, near-duplicates are removed (MinHash), rows
that mention a held-out task are dropped (decontamination), sources are
weighted and capped, and an optional general-text replay slice is mixed in
against forgetting. Only text source files are read (extensions on an allow
list, NUL bytes rejected); no compiled artefact is opened.

    python -m kore_b200.data.midtrain_corpus --out corpus.jsonl [--max-docs 20000]

Output rows: {"text", "source", "path"} (the midtrain trainer reads "text").
Reference parity: kore/data/midtrain_corpus.py (sources, chunking, near-dedup,
held-out exclusion, source weights, general replay), with B200 sources.
"""
from __future__ import annotations

import argparse
import inspect
import json
import os
import random
import re
import site
import sys
from collections import Counter
from pathlib import Path
from typing import Dict, Iterable, Iterator, List, Optional, Sequence

from .corpus_quality import CODE_EXT, DOC_EXT, quality_filter
from .hygiene import dedup

ROOT = Path(__file__).resolve().parents[2]
SOURCE_WEIGHTS = {"tasks": 1.0, "repo_kernels": 1.0, "cutlass": 0.6, "triton": 0.8, "docs": 0.5, "wins": 1.0}
_SKIP_DIRS = {"__pycache__", ".git", "test", "tests", "testing", "build", "dist", "node_modules", "examples_data"}
_MAX_FILE = 400_000


def chunk_text(text: str, budget: int) -> List[str]:
    """Cut ``text`` into pieces of at most ``budget`` characters at line
    boundaries (a single longer line becomes its own piece, truncated)."""
    out, cur, n = [], [], 0
    for ln in text.splitlines(keepends=True):
        if n + len(ln) > budget and cur:
            out.append("".join(cur))
            cur, n = [], 0
        cur.append(ln[:budget])
        n += min(len(ln), budget)
    if cur:
        out.append("".join(cur))
    return [c for c in out if c.strip()]


def _read(path: Path) -> Optional[str]:
    try:
        if path.stat().st_size > _MAX_FILE:
            return None
        raw = path.read_bytes()
    except OSError:
        return None
    if b"\x00" in raw[:8192]:
        return None
    try:
        return raw.decode("utf-8")
    except UnicodeDecodeError:
        return None


def _walk(root: Path, exts: Iterable[str], limit: int) -> Iterator[Path]:
    exts = set(exts)
    n = 0
    for dirpath, dirnames, filenames in os.walk(root):
        dirnames[:] = sorted(d for d in dirnames if d not in _SKIP_DIRS and not d.startswith("."))
        for f in sorted(filenames):
            if Path(f).suffix.lower() in exts:
                yield Path(dirpath) / f
                n += 1
                if n >= limit:
                    return


def site_roots() -> List[Path]:
    roots = []
    for p in list(site.getsitepackages()) + [site.getusersitepackages()] + sys.path:
        q = Path(p)
        if q.is_dir() and q.name in ("site-packages", "dist-packages") and q not in roots:
            roots.append(q)
    return roots


def cutlass_roots() -> List[Path]:
    """CUTLASS / CuTe include trees shipped inside installed packages."""
    out = []
    for sp in site_roots():
        for cand in sp.glob("*/data/cutlass/include") or []:
            out.append(cand)
        for cand in sp.glob("*/3rdparty/cutlass/include") or []:
            out.append(cand)
    seen, uniq = set(), []
    for p in out:
        r = p.resolve()
        if r not in seen:
            seen.add(r)
            uniq.append(p)
    return uniq


# ---------------------------------------------------------------- sources
def task_docs(heldout: Sequence[str] = ()) -> List[dict]:
    from ..tasks.ops_library import SPECS
    from ..tasks.registry import all_tasks
    held = set(heldout)
    rows = []
    for t in all_tasks():
        if t.task_id in held:
            continue
        spec = SPECS.get(getattr(t, "spec", t.task_id))
        ref = ""
        if spec is not None:
            try:
                ref = inspect.getsource(spec.reference)
            except (OSError, TypeError):
                ref = ""
        text = (f"# {t.task_id}: {t.operation} ({t.dtype})\n\n"
                + (f"Oracle:\n```python\n{ref}```\n\n" if ref else "")
                + f"Seed kernel:\n```python\n{t.seed_src}\n```\n")
        rows.append({"text": text, "source": "tasks", "path": t.task_id, "kind": "record"})
    return rows


def repo_kernel_docs() -> List[dict]:
    rows = []
    for sub in ("kore_b200/csrc", "kore_b200/ops"):
        for p in _walk(ROOT / sub, CODE_EXT, 200):
            t = _read(p)
            if t:
                rows.append({"text": t, "source": "repo_kernels", "path": str(p.relative_to(ROOT)), "kind": "code"})
    return rows


def cutlass_docs(limit: int = 3000) -> List[dict]:
    rows = []
    for root in cutlass_roots():
        files = list(_walk(root, {".h", ".hpp", ".cuh", ".inl"}, limit))
        files.sort(key=lambda p: (0 if re.search(r"sm100|tcgen05|umma|tmem|blackwell", str(p), re.I) else 1, str(p)))
        for p in files[:limit]:
            t = _read(p)
            if t:
                rows.append({"text": t, "source": "cutlass", "path": str(p), "kind": "code"})
    return rows


def triton_docs(limit: int = 2000) -> List[dict]:
    rows = []
    for sp in site_roots():
        for pkg in ("triton", "flashinfer", "vllm", "flash_attn"):
            root = sp / pkg
            if not root.is_dir():
                continue
            for p in _walk(root, {".py"}, limit):
                t = _read(p)
                if t and "@triton.jit" in t:
                    rows.append({"text": t, "source": "triton", "path": str(p), "kind": "code"})
    return rows


def doc_docs(limit: int = 500) -> List[dict]:
    rows = []
    pb = ROOT / "kore_b200" / "data" / "knowledge" / "b200_playbook.md"
    t = _read(pb)
    if t:
        rows.append({"text": t, "source": "docs", "path": str(pb.relative_to(ROOT)), "kind": "doc"})
    for root in cutlass_roots():
        base = root.parent
        for p in _walk(base, DOC_EXT, limit):
            t = _read(p)
            if t:
                rows.append({"text": t, "source": "docs", "path": str(p), "kind": "doc"})
    return rows


def win_docs(wins: Iterable) -> List[dict]:
    rows = []
    for w in wins:
        k = getattr(w, "final_kernel", None)
        if k:
            rows.append({"text": f"# Optimised kernel for {w.task_id} ({(w.speedup or 0):.2f}x over the seed)\n\n"
                                 f"```python\n{k}\n```\n", "source": "wins", "path": w.task_id, "kind": "record"})
    return rows


# ---------------------------------------------------------------- assembly
def mentions_heldout(text: str, heldout: Sequence[str]) -> bool:
    return any(h in text for h in heldout if len(h) >= 8)


def build_midtrain_corpus(out_path: Optional[str] = None, *, wins: Iterable = (), max_docs: int = 20000,
                          chunk_chars: int = 16000, dedup_threshold: float = 0.8, general_replay: str = "",
                          replay_frac: float = 0.1, seed: int = 0, sources: Optional[Sequence[str]] = None,
                          weights: Optional[Dict[str, float]] = None) -> Dict[str, object]:
    from ..tasks.registry import split_tasks
    _, heldout = split_tasks()
    want = set(sources or SOURCE_WEIGHTS)
    collectors = {"tasks": lambda: task_docs(heldout), "repo_kernels": repo_kernel_docs, "cutlass": cutlass_docs,
                  "triton": triton_docs, "docs": doc_docs, "wins": lambda: win_docs(wins)}
    raw: List[dict] = []
    for name, fn in collectors.items():
        if name in want:
            raw += fn()
    kept, reasons = quality_filter(raw)
    chunks = []
    for r in kept:
        for i, c in enumerate(chunk_text(r["text"], chunk_chars)):
            chunks.append({"text": c, "source": r["source"], "path": r["path"] + (f"#{i}" if i else "")})
    n_before = len(chunks)
    chunks = [c for c in chunks if not mentions_heldout(c["text"], heldout)]
    decontaminated = n_before - len(chunks)
    chunks = dedup(chunks, key=lambda r: r["text"][:4000], threshold=dedup_threshold)
    rng = random.Random(seed)
    w = dict(SOURCE_WEIGHTS, **(weights or {}))
    by_src: Dict[str, List[dict]] = {}
    for c in chunks:
        by_src.setdefault(c["source"], []).append(c)
    tot_w = sum(w.get(s, 0.5) for s in by_src) or 1.0
    budget = int(max_docs * (1.0 - (replay_frac if general_replay else 0.0)))
    out: List[dict] = []
    for s, rows in sorted(by_src.items()):
        rng.shuffle(rows)
        out += rows[: max(1, int(budget * w.get(s, 0.5) / tot_w))]
    if general_replay and os.path.exists(general_replay):
        from .datasets import load_text_rows
        txt = load_text_rows(general_replay)
        rng.shuffle(txt)
        n = int(max_docs * replay_frac)
        out += [{"text": t, "source": "general_replay", "path": general_replay} for t in txt[:n]]
    rng.shuffle(out)
    counts = Counter(r["source"] for r in out)
    if out_path:
        Path(out_path).parent.mkdir(parents=True, exist_ok=True)
        with open(out_path, "w") as f:
            for r in out:
                f.write(json.dumps(r) + "\n")
    return {"docs": len(out), "by_source": dict(counts), "raw": len(raw), "quality_drops": reasons,
            "decontaminated": decontaminated, "chunks_before_dedup": n_before, "rows": out}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore midtrain-corpus")
    ap.add_argument("--out", required=True)
    ap.add_argument("--max-docs", type=int, default=20000)
    ap.add_argument("--chunk-chars", type=int, default=16000)
    ap.add_argument("--sources", default="")
    ap.add_argument("--general-replay", default="")
    ap.add_argument("--wins", default="", help="win-record JSONL files")
    a = ap.parse_args(argv)
    wins = []
    if a.wins:
        from .schemas import WinRecord, read_records
        for p in a.wins.split(","):
            wins += list(read_records(p, WinRecord))
    rep = build_midtrain_corpus(a.out, wins=wins, max_docs=a.max_docs, chunk_chars=a.chunk_chars,
                                general_replay=a.general_replay,
                                sources=[s for s in a.sources.split(",") if s] or None)
    rep.pop("rows")
    print(json.dumps(rep))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
