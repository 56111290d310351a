#!/usr/bin/env python3
"""Shape-specialised OptimizerSettings, generated from measured sweeps.

Same interface and rules as the reference's ``src/dispatch.py`` (:1-260):
``shape_key`` / ``load_table`` / ``lookup`` / ``applicable_settings`` /
``build_entries`` and a generator CLI. The records come from this build's
appendix sweep (``bench.py --sweep ... [--set field=value ...]``, one JSON
line per shape carrying the shape, the median forward time and the
``OptimizerSettings`` it ran with); the generator keeps the fastest record
per shape and writes the table, and ``settings_for(config)`` applies it.

    python transformer-kernel_b200/sweep.py model --out model.jsonl
    python transformer-kernel_b200/sweep.py gemm --out gemm.jsonl
    python transformer-kernel_b200/dispatch.py model.jsonl --gemm gemm.jsonl --out dispatch.json

(``bench.py --sweep`` lines are accepted as model records too.) The table
also carries ``gemm_tiles``: per measured GEMM shape (M, N, K, epilogue) the
fastest tile variant whose output agreed with the built-in choice; the
drop-in pushes them into ``libtk_b200`` (``tk_gemm_tiles_set``) once per
process, where ``tk_gemm`` consults them before its built-in rules.

Rules (as in the reference):
  * only ``OptimizerSettings`` fields are applied; other keys stay in the
    table for provenance;
  * explicitly chosen fields beat the table (``explicit``);
  * medians from different sweep files were taken on different boxes and
    clocks: cross-file wins within a few percent are ties.
Unlike the reference's settings, none of these select another backend or a
lower precision: every combination runs the same B200 kernels with the same
numerics (the test suite checks each path against the oracle), so the table
only trades speed.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import pathlib
import time
from typing import Dict, Iterable, Optional

HERE = pathlib.Path(__file__).resolve().parent
DEFAULT_TABLE_PATH = HERE / "dispatch.json"

SHAPE_FIELDS = ("batch_size", "seq_len", "d_model", "heads", "layers", "ffn_dim", "causal")

# bench.py --sweep shape names -> SHAPE_FIELDS
_SWEEP_SHAPE = {"batch": "batch_size", "seq": "seq_len", "d_model": "d_model", "heads": "heads",
                "layers": "layers", "ffn": "ffn_dim", "causal": "causal"}


def shape_key(batch_size: int, seq_len: int, d_model: int, heads: int, layers: int, ffn_dim: int,
              causal: bool) -> str:
    suffix = "causal" if causal else "bidir"
    return f"b{batch_size}-s{seq_len}-d{d_model}-h{heads}-l{layers}-f{ffn_dim}-{suffix}"


def config_shape(config) -> Dict[str, object]:
    """SHAPE_FIELDS of a harness-style TransformerConfig."""
    return {"batch_size": config.batch_size, "seq_len": config.seq_len, "d_model": config.d_model,
            "heads": config.num_heads, "layers": config.num_layers, "ffn_dim": config.ffn_dim,
            "causal": bool(config.causal)}


def load_table(path: Optional[pathlib.Path] = None) -> Optional[dict]:
    path = DEFAULT_TABLE_PATH if path is None else pathlib.Path(path)
    if not path.exists():
        return None
    return json.loads(path.read_text())


def lookup(table: dict, **shape) -> Optional[dict]:
    """The measured entry whose key is this shape's (fields as in
    SHAPE_FIELDS), or None when the sweep never ran the shape."""
    return (table.get("entries") or {}).get(shape_key(**shape))


def _field_types() -> Dict[str, type]:
    from optimized import OptimizerSettings

    return {f.name: (bool if f.type in ("bool", bool) else str) for f in dataclasses.fields(OptimizerSettings)}


def applicable_settings(entry_settings: Dict[str, object], explicit: Iterable[str] = ()) -> Dict[str, object]:
    """The table settings that are OptimizerSettings fields and were not set
    explicitly, coerced to the field types."""
    valid = _field_types()
    explicit = set(explicit)
    applied = {}
    for key, value in entry_settings.items():
        if key not in valid or key in explicit:
            continue
        if valid[key] is bool and isinstance(value, str):
            value = value == "True"
        applied[key] = value
    return applied


def settings_for(config, table: Optional[dict] = None, base=None, explicit: Iterable[str] = ()):
    """OptimizerSettings for `config`: `base` (default: the active settings)
    with the table's entry for the shape applied, if there is one."""
    import optimized

    base = optimized.active_settings() if base is None else base
    table = load_table() if table is None else table
    entry = lookup(table, **config_shape(config)) if table else None
    if not entry:
        return base
    return dataclasses.replace(base, **applicable_settings(entry.get("settings") or {}, explicit))


def _records(path: pathlib.Path):
    """Sweep records of a JSON-lines file: ``bench.py --sweep`` lines as they
    are, ``sweep.py`` case lines unwrapped (only cases that ran to the end;
    records that failed their accuracy check are dropped)."""
    for line in path.read_text().splitlines():
        line = line.strip()
        if not line.startswith("{"):
            continue
        try:
            item = json.loads(line)
        except ValueError:
            continue
        if "records" in item:
            if item.get("status") not in ("ok", "accuracy_failed"):
                continue
            for rec in item["records"]:
                if rec.get("status", "ok") == "ok":
                    yield rec
        elif item.get("status", "ok") == "ok":
            yield item


def build_entries(paths: Iterable[pathlib.Path]) -> Dict[str, dict]:
    """Fastest sweep record per shape over JSON-line files written by
    ``sweep.py model`` or ``bench.py --sweep``."""
    entries: Dict[str, dict] = {}
    for path in paths:
        path = pathlib.Path(path)
        for record in _records(path):
            ms, settings, shape = record.get("ms"), record.get("settings"), record.get("shape")
            if ms is None or not settings or not shape:
                continue
            try:
                key = shape_key(**{_SWEEP_SHAPE[k]: shape[k] for k in _SWEEP_SHAPE})
            except KeyError:
                continue
            best = entries.get(key)
            if best is None or ms < best["median_ms"]:
                entries[key] = {"settings": settings, "median_ms": ms, "path": record.get("path"),
                                "source": path.name, "case_id": record.get("case")}
    return dict(sorted(entries.items()))


TILE_TIE = 0.03  # a variant must beat the built-in choice by more than this fraction
# GEMMs at or below this M*N*K are launch-bound: the library launches them
# with programmatic dependent launch, overlapped with their neighbours, so
# their isolated back-to-back timing does not predict their time inside a
# forward (measured: C2 forward 0.213 -> 0.244 ms with isolated-sweep picks).
# They keep the built-in choice.
SMALL_GEMM_MNK = 8.6e9


def build_gemm_tiles(paths: Iterable[pathlib.Path]) -> list:
    """Fastest accepted tile variant per GEMM shape (M, N, K, epilogue) over
    ``sweep.py gemm`` files, with every variant's time for provenance. A
    variant within TILE_TIE of the built-in choice ("auto") is a tie and
    leaves the built-in choice in place (launch-time noise is a few percent)."""
    best: Dict[tuple, dict] = {}
    for path in paths:
        for rec in _records(pathlib.Path(path)):
            if "variant" not in rec or rec.get("ms") is None:
                continue
            key = (rec["M"], rec["N"], rec["K"], rec["epilogue"])
            entry = best.setdefault(key, {"M": rec["M"], "N": rec["N"], "K": rec["K"], "epilogue": rec["epilogue"],
                                          "gemm": rec.get("gemm"), "shape_name": rec.get("shape_name"),
                                          "variant": None, "ms": None, "alternatives": {}})
            entry["alternatives"][rec["variant"]] = round(rec["ms"], 5)
            if entry["ms"] is None or rec["ms"] < entry["ms"]:
                entry["variant"], entry["ms"] = rec["variant"], rec["ms"]
    for entry in best.values():
        auto = entry["alternatives"].get("auto")
        small = float(entry["M"]) * entry["N"] * entry["K"] <= SMALL_GEMM_MNK
        if auto is not None and (small or entry["ms"] > (1.0 - TILE_TIE) * auto):
            entry["variant"], entry["ms"] = "auto", auto
            if small:
                entry["note"] = "launch-bound: built-in choice kept"
    return [best[k] for k in sorted(best)]


_APPLIED = False


def apply_gemm_tiles(table: Optional[dict]) -> int:
    """Push the table's GEMM tile choices into the library (replacing any
    there); returns the number of entries set."""
    import _tklib as tk
    import linear

    tk.lib().tk_gemm_tiles_clear()
    n = 0
    for e in (table or {}).get("gemm_tiles") or []:
        if e.get("variant") is None:
            continue
        # built-in ("auto") choices are entries too: a measured M that kept the
        # built-in choice must be the nearest match for the Ms around it
        tk.call("tk_gemm_tiles_set", e["M"], e["N"], e["K"], linear.EPILOGUES[e["epilogue"]], tk.TILES[e["variant"]])
        n += 1
    return n


def ensure_applied() -> None:
    """Once per process: the packaged table's GEMM tile choices go to the
    library (called by the drop-in when it first builds its weights)."""
    global _APPLIED
    if not _APPLIED:
        _APPLIED = True
        apply_gemm_tiles(load_table())


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("results", nargs="*", help="model sweep records (sweep.py model, bench.py --sweep)")
    parser.add_argument("--gemm", nargs="*", default=[], help="GEMM sweep records (sweep.py gemm)")
    parser.add_argument("--out", default=str(DEFAULT_TABLE_PATH))
    args = parser.parse_args()
    paths = [pathlib.Path(p) for p in args.results]
    gpaths = [pathlib.Path(p) for p in args.gemm]
    entries = build_entries(paths)
    tiles = build_gemm_tiles(gpaths)
    if not entries and not tiles:
        print("no sweep records found in the given files")
        return 1
    payload = {"schema": 2, "generated_at": time.strftime("%Y-%m-%dT%H:%M:%S%z"),
               "sources": [p.name for p in paths + gpaths], "entries": entries, "gemm_tiles": tiles}
    out = pathlib.Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(payload, indent=2) + "\n")
    width = max([len(k) for k in entries] or [1])
    for key, entry in entries.items():
        print(f"{key:<{width}}  {entry['median_ms']:>9.4f} ms  {entry['settings']}  <- {entry['source']}")
    for t in tiles:
        print(f"gemm {t['M']}x{t['N']}x{t['K']} {t['epilogue']}: {t['variant']} {t['ms']:.4f} ms  {t['alternatives']}")
    print(f"\nwrote {out} ({len(entries)} shapes, {len(tiles)} GEMM shapes)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
