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


# ---- the per-shape sweep runner and the GEMM tile table ---------------------

import stat  # noqa: E402

import pytest  # noqa: E402

import sweep  # noqa: E402


def _fake_python(tmp_path, body):
    """A stand-in interpreter for the runner's child: ignores its arguments."""
    p = tmp_path / "fake_python.sh"
    p.write_text("#!/bin/sh\n" + body + "\n")
    p.chmod(p.stat().st_mode | stat.S_IEXEC)
    return str(p)


@pytest.mark.parametrize("body,status", [
    ("echo '{\"variant\": \"pair\", \"ms\": 1.5}'; exit 0", "ok"),
    ("echo '{\"variant\": \"pair\", \"ms\": 1.5, \"status\": \"accuracy_failed\"}'; exit 2", "accuracy_failed"),
    ("echo boom >&2; exit 1", "error"),
    ("sleep 5", "timeout"),
])
def test_run_case_classifies_like_the_reference(tmp_path, body, status):
    res = sweep.run_case("gemm", "C2", timeout=0.5 if status == "timeout" else 60,
                         python=_fake_python(tmp_path, body))
    assert res["status"] == status and res["case"] == "C2"
    if status == "ok":
        assert res["records"] == [{"variant": "pair", "ms": 1.5}]
    if status == "error":
        assert "boom" in res["stderr_tail"]


def test_gemm_shapes_follow_the_forward():
    got = {g["gemm"]: (g["M"], g["N"], g["K"], g["epilogue"]) for g in sweep.gemm_shapes("C3")}
    assert got == {"qkv": (65536, 3072, 1024, "bias"), "ffn_in": (65536, 4096, 1024, "gelu"),
                   "o": (65536, 1024, 1024, "resid"), "ffn_out": (65536, 1024, 4096, "resid")}
    # d_model 128 fuses its LayerNorm in one tile: no tile choice for O / FFN-out
    assert {g["gemm"] for g in sweep.gemm_shapes("13")} == {"qkv", "ffn_in"}
    # the out-of-core-scale shape is measured at a bounded M
    assert all(g["M"] == sweep.GEMM_MAX_M for g in sweep.gemm_shapes("C5"))


def test_build_gemm_tiles_keeps_the_fastest_accepted_variant(tmp_path):
    rec = lambda v, ms, st="ok": {"gemm": "qkv", "M": 4096, "N": 3072, "K": 1024, "epilogue": "bias",  # noqa: E731
                                  "shape_name": "C3", "variant": v, "ms": ms, "status": st}
    f = tmp_path / "g.jsonl"
    f.write_text(json.dumps({"kind": "gemm", "case": "C3", "status": "accuracy_failed",
                             "records": [rec("auto", 1.0), rec("pair", 0.8), rec("bn64", 0.5, "accuracy_failed")]})
                 + "\n" + json.dumps({"kind": "gemm", "case": "C3b", "status": "ok",
                                       "records": [dict(rec("auto", 2.0), M=8192), dict(rec("bn128", 1.98), M=8192)]})
                 + "\n" + json.dumps({"kind": "gemm", "case": "X", "status": "timeout", "records": [rec("bn128", 0.1)]})
                 + "\n")
    tiles = {t["M"]: t for t in dispatch.build_gemm_tiles([f])}
    assert len(tiles) == 2
    assert tiles[4096]["variant"] == "pair" and tiles[4096]["alternatives"] == {"auto": 1.0, "pair": 0.8}
    assert tiles[8192]["variant"] == "auto"  # 1% faster is a tie: the built-in choice stays
    small = tmp_path / "small.jsonl"
    small.write_text(json.dumps({"kind": "gemm", "case": "C2", "status": "ok",
                                 "records": [dict(rec("auto", 1.0), M=512), dict(rec("bn64", 0.5), M=512)]}) + "\n")
    # 512 x 3072 x 1024 is launch-bound: the isolated winner does not replace the built-in choice
    assert dispatch.build_gemm_tiles([small])[0]["variant"] == "auto"


def test_apply_gemm_tiles_fills_the_library_table():
    import _tklib as tk

    table = {"gemm_tiles": [{"M": 4096, "N": 3072, "K": 1024, "epilogue": "bias", "variant": "pair"},
                            {"M": 512, "N": 512, "K": 512, "epilogue": "resid", "variant": "auto"}]}
    try:
        assert dispatch.apply_gemm_tiles(table) == 2  # the built-in choice is an entry too
        with pytest.raises(tk.TKError):
            tk.call("tk_gemm_tiles_set", 0, 1, 1, 0, 1)  # a bad entry is refused on the host
    finally:
        tk.lib().tk_gemm_tiles_clear()
