"""Per-shape settings dispatch (CPU): the same shape keys, lookup and
coercion rules as the reference's src/dispatch.py, over this build's sweep
records (bench.py --sweep JSON lines)."""

from __future__ import annotations

import json

import dispatch
import optimized


def _record(case, ms, **settings):
    base = {"fused_ln_epilogue": True, "assume_dense_mask": False, "check_device_errors": False,
            "fused_small_stack": True}
    base.update(settings)
    return {"case": case, "shape": {"batch": 64, "seq": 128, "d_model": 128, "heads": 4, "ffn": 128, "layers": 4,
                                    "causal": True}, "ms": ms, "settings": base}


def test_shape_key_matches_the_reference_format():
    assert dispatch.shape_key(64, 128, 128, 4, 4, 128, True) == "b64-s128-d128-h4-l4-f128-causal"
    assert dispatch.shape_key(256, 256, 1024, 16, 4, 4096, False) == "b256-s256-d1024-h16-l4-f4096-bidir"


def test_build_entries_keeps_the_fastest_record(tmp_path):
    a, b = tmp_path / "a.jsonl", tmp_path / "b.jsonl"
    a.write_text(json.dumps(_record(1, 0.12)) + "\nnot json\n")
    b.write_text(json.dumps(_record(1, 0.20, fused_small_stack=False)) + "\n")
    entries = dispatch.build_entries([a, b])
    entry = entries["b64-s128-d128-h4-l4-f128-causal"]
    assert entry["median_ms"] == 0.12 and entry["settings"]["fused_small_stack"] is True and entry["source"] == "a.jsonl"


def test_settings_for_applies_the_entry_but_not_explicit_fields():
    table = {"entries": {"b64-s128-d128-h4-l4-f128-causal": {
        "settings": {"fused_small_stack": "False", "fused_ln_epilogue": False, "unknown_field": 3}}}}
    cfg = optimized.TransformerConfig(64, 128, 128, 4, 128, 4, True)
    s = dispatch.settings_for(cfg, table, base=optimized.OptimizerSettings())
    assert s.fused_small_stack is False and s.fused_ln_epilogue is False
    s2 = dispatch.settings_for(cfg, table, base=optimized.OptimizerSettings(), explicit={"fused_small_stack"})
    assert s2.fused_small_stack is True and s2.fused_ln_epilogue is False
    other = optimized.TransformerConfig(1, 512, 512, 8, 2048, 4, True)
    assert dispatch.settings_for(other, table, base=optimized.OptimizerSettings()) == optimized.OptimizerSettings()


def test_generator_cli_writes_a_loadable_table(tmp_path):
    src, out = tmp_path / "s.jsonl", tmp_path / "t.json"
    src.write_text(json.dumps(_record(1, 0.1)) + "\n")
    import sys
    argv = sys.argv
    try:
        sys.argv = ["dispatch.py", str(src), "--out", str(out)]
        assert dispatch.main() == 0
    finally:
        sys.argv = argv
    table = dispatch.load_table(out)
    assert dispatch.lookup(table, batch_size=64, seq_len=128, d_model=128, heads=4, layers=4, ffn_dim=128,
                           causal=True)["median_ms"] == 0.1
