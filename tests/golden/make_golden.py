#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle.

Run in a container that holds the reference checkout (the harness is plain
PyTorch, so it runs on the CPU unmodified):

    python tests/golden/make_golden.py --reference-src <checkout>/src

For every case it imports the organisers' harness
``src/torch_transformer_benchmark.py`` as-is, builds ``BaselineTransformer``
under ``torch.manual_seed(0)`` (default init), draws the input with the
harness's own ``generate_random_case`` on the CPU and runs the fp32 forward.
It stores, per case, a checksum of every weight, the input checksum, and the
output -- whole for small cases, as per-token row sums plus a few full
token rows for the larger ones -- in ``golden.pt`` next to this script.
Fixtures are small (well under 2 MB in total).

Nothing at test time reads the reference checkout; the tests only read the
fixture file.
"""

from __future__ import annotations

import argparse
import importlib.util
import pathlib
import sys

import torch

HERE = pathlib.Path(__file__).resolve().parent

# (name, B, S, d, H, ffn, L, causal, padding_ratio, input_seed, keep_full)
CASES = [
    ("tiny_causal", 2, 16, 64, 4, 128, 2, True, 0.0, 1234, True),
    ("tiny_bidir", 2, 16, 64, 4, 128, 2, False, 0.0, 1235, True),
    ("tiny_padded", 3, 24, 64, 4, 128, 2, True, 0.3, 1236, True),
    ("ragged_s", 2, 100, 128, 4, 256, 1, True, 0.0, 1237, True),
    ("c1_reference_case1", 64, 128, 128, 4, 128, 4, True, 0.0, 1234, False),
    ("c2_small_batch", 1, 512, 512, 8, 2048, 4, True, 0.0, 1234, False),
    ("c3_slice_b2_l1", 2, 256, 1024, 16, 4096, 1, False, 0.0, 1234, False),
    ("c4_slice_s1024_l1", 1, 1024, 1024, 16, 4096, 1, True, 0.0, 1234, False),
]

KEEP_ROWS = 4  # full token rows kept for large cases: first and last of batch 0 and B-1


def load_harness(src: pathlib.Path):
    spec = importlib.util.spec_from_file_location(
        "torch_transformer_benchmark", src / "torch_transformer_benchmark.py"
    )
    module = importlib.util.module_from_spec(spec)
    sys.modules["torch_transformer_benchmark"] = module
    spec.loader.exec_module(module)
    return module


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference-src", required=True, type=pathlib.Path)
    parser.add_argument("--out", type=pathlib.Path, default=HERE / "golden.pt")
    args = parser.parse_args()

    bench = load_harness(args.reference_src)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    fixtures = {}
    for name, b, s, d, h, f, layers, causal, pad, seed, keep_full in CASES:
        cfg = bench.TransformerConfig(b, s, d, h, f, layers, causal)
        cfg.validate()
        torch.manual_seed(0)
        model = bench.BaselineTransformer(cfg).eval()
        x, mask = bench.generate_random_case(
            cfg, torch.device("cpu"), torch.float32, seed, pad, 1.0
        )
        with torch.inference_mode():
            out = model(x, mask)
        entry = {
            "config": dict(batch_size=b, seq_len=s, d_model=d, num_heads=h, ffn_dim=f,
                           num_layers=layers, causal=causal),
            "padding_ratio": pad,
            "input_seed": seed,
            "weight_checksums": {k: (float(v.double().sum()), float(v.double().abs().sum()))
                                 for k, v in model.state_dict().items()},
            "weight_keys": list(model.state_dict().keys()),
            "x_checksum": (float(x.double().sum()), float(x.double().abs().sum())),
            "mask": mask.clone(),
            "out_row_sums": out.double().sum(-1).float().clone(),
            "out_abs_sum": float(out.double().abs().sum()),
        }
        if keep_full:
            entry["out"] = out.clone()
        else:
            rows = [(0, 0), (0, s - 1), (b - 1, 0), (b - 1, s - 1)][:KEEP_ROWS]
            entry["out_rows_index"] = rows
            entry["out_rows"] = torch.stack([out[i, j] for i, j in rows]).clone()
        fixtures[name] = entry
        print(f"{name}: out abs sum {entry['out_abs_sum']:.6f}")
    fixtures["_meta"] = {"torch": torch.__version__, "generator": "tests/golden/make_golden.py"}
    torch.save(fixtures, args.out)
    print(f"wrote {args.out} ({args.out.stat().st_size / 1e6:.2f} MB)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
