#!/usr/bin/env python3
"""Shape-specialised OptimizerSettings, generated from measured sweeps.

Same interface and rules as the reference's ``src/dispatch.py`` (:1-260):
``shape_key`` / ``load_table`` / ``lookup`` / ``applicable_settings`` /
``build_entries`` and a generator CLI. The records come from this build's
appendix sweep (``bench.py --sweep ... [--set field=value ...]``, one JSON
line per shape carrying the shape, the median forward time and the
``OptimizerSettings`` it ran with); the generator keeps the fastest record
per shape and writes the table, and ``settings_for(config)`` applies it.

    python bench.py --sweep all > a.jsonl
    python bench.py --sweep all --set fused_small_stack=False > b.jsonl
    python transformer-kernel_b200/dispatch.py a.jsonl b.jsonl --out dispatch.json

Rules (as in the reference):
  * only ``OptimizerSettings`` fields are applied; other keys stay in the
    table for provenance;
  * explicitly chosen fields beat the table (``explicit``);
  * medians from different sweep files were taken on different boxes and
    clocks: cross-file wins within a few percent are ties.
Unlike the reference's settings, none of these select another backend or a
lower precision: every combination runs the same B200 kernels with the same
numerics (the test suite checks each path against the oracle), so the table
only trades speed. The library's own tile choices (GEMM tile width, CTA-pair
kernel, programmatic launch) are made per call inside ``libtk_b200``.
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
    """Table entry for a shape given as SHAPE_FIELDS keyword arguments."""
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


def build_entries(paths: Iterable[pathlib.Path]) -> Dict[str, dict]:
    """Fastest sweep record per shape over JSON-line files written by
    ``bench.py --sweep``."""
    entries: Dict[str, dict] = {}
    for path in paths:
        path = pathlib.Path(path)
        for line in path.read_text().splitlines():
            line = line.strip()
            if not line.startswith("{"):
                continue
            record = json.loads(line)
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


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("results", nargs="+", help="JSON-line files written by bench.py --sweep")
    parser.add_argument("--out", default=str(DEFAULT_TABLE_PATH))
    args = parser.parse_args()
    paths = [pathlib.Path(p) for p in args.results]
    entries = build_entries(paths)
    if not entries:
        print("no sweep records found in the given files")
        return 1
    payload = {"schema": 1, "generated_at": time.strftime("%Y-%m-%dT%H:%M:%S%z"),
               "sources": [p.name for p in paths], "entries": entries}
    out = pathlib.Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(payload, indent=2) + "\n")
    width = max(len(k) for k in entries)
    for key, entry in entries.items():
        print(f"{key:<{width}}  {entry['median_ms']:>9.4f} ms  {entry['settings']}  <- {entry['source']}")
    print(f"\nwrote {out} ({len(entries)} shapes from {len(paths)} files)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
