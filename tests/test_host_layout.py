"""Host-side layout checks (CPU, no GPU needed): the packed per-layer weight
and vector buffers that tk_stack_small reads (include/tk_b200.h: rows Wq, Wk,
Wv, Wo, W_in, W_out per layer; vector bq|bk|bv, bo, b_in, b_out, norm1 w/b,
norm2 w/b) are assembled from the harness's module tree in that order."""

from __future__ import annotations

import torch

import optimized
from oracle import StackConfig, init_params


def test_small_stack_packing_layout():
    cfg = StackConfig(2, 16, 128, 4, 128, 3, True)
    params = init_params(cfg, seed=0)
    model = optimized.OptimizedTransformer(cfg)
    model.load_state_dict(params, strict=True)
    weights = model._weights()
    w, vec, eps = model._small_stack_pack(weights)
    assert w.dtype == torch.float16 and tuple(w.shape) == (3 * 768, 128)
    assert vec.dtype == torch.float32 and tuple(vec.shape) == (3, 1280)
    assert eps == 1e-5
    for i in range(cfg.num_layers):
        p = lambda name: params[f"layers.{i}.{name}"]  # noqa: E731
        rows = w[i * 768:(i + 1) * 768].float()
        for off, name in [(0, "attention.q_proj"), (128, "attention.k_proj"), (256, "attention.v_proj"),
                          (384, "attention.out_proj"), (512, "ffn_in"), (640, "ffn_out")]:
            torch.testing.assert_close(rows[off:off + 128], p(f"{name}.weight").half().float(), atol=0, rtol=0)
        v = vec[i]
        for off, name in [(0, "attention.q_proj.bias"), (128, "attention.k_proj.bias"), (256, "attention.v_proj.bias"),
                          (384, "attention.out_proj.bias"), (512, "ffn_in.bias"), (640, "ffn_out.bias"),
                          (768, "norm1.weight"), (896, "norm1.bias"), (1024, "norm2.weight"), (1152, "norm2.bias")]:
            torch.testing.assert_close(v[off:off + 128], p(name), atol=0, rtol=0)


def test_small_stack_declines_mixed_layernorm_eps():
    cfg = StackConfig(1, 8, 128, 4, 128, 2, True)
    model = optimized.OptimizedTransformer(cfg)
    model.load_state_dict(init_params(cfg, seed=0), strict=True)
    model.layers[1].norm2.eps = 1e-6
    assert model._small_stack_pack(model._weights()) is None


def test_state_dict_reload_rebuilds_the_weight_cache():
    # load_state_dict copies into the existing parameters (same storage), so
    # the derived fp16 copies must be rebuilt from the new values.
    cfg = StackConfig(1, 8, 128, 4, 128, 2, True)
    model = optimized.OptimizedTransformer(cfg)
    model.load_state_dict(init_params(cfg, seed=0), strict=True)
    first = model._weights()
    model._small_stack_pack(first)
    ptr = model.layers[0].attention.q_proj.weight.data_ptr()
    fresh = init_params(cfg, seed=1)
    model.load_state_dict(fresh, strict=True)
    assert model.layers[0].attention.q_proj.weight.data_ptr() == ptr
    again = model._weights()
    assert again is not first
    want = torch.cat([fresh[f"layers.1.attention.{n}_proj.weight"] for n in "qkv"], 0).half()
    torch.testing.assert_close(again[1].qkv_w, want, atol=0, rtol=0)
    w, _, _ = model._small_stack_pack(again)
    torch.testing.assert_close(w[768:768 + 384], want, atol=0, rtol=0)


def test_state_dict_reload_drops_captured_graphs():
    import cuda_graphs

    cfg = StackConfig(1, 8, 128, 4, 128, 2, True)
    model = cuda_graphs.GraphedTransformer(cfg)
    model.load_state_dict(init_params(cfg, seed=0), strict=True)
    model._graph_states[("shape",)] = cuda_graphs._GraphState()
    model.load_state_dict(init_params(cfg, seed=1), strict=True)
    assert model._graph_states == {}


def test_forward_paths_are_opaque_to_torch_compile():
    # the harness may torch.compile the drop-in (--compile-user); every entry
    # point runs eagerly inside a compiled caller
    import cuda_graphs
    import sharded

    for fn in (optimized.OptimizedTransformer.forward, optimized.OptimizedTransformer.forward_from_host,
               optimized.OptimizedTransformer._weights, optimized.OptimizedTransformer._prefix_lengths,
               cuda_graphs.GraphedTransformer.forward, sharded.ShardedTransformer.forward):
        assert getattr(fn, "_torchdynamo_disable", False), fn


def test_compiled_model_runs_the_eager_forward():
    # torch.compile around the drop-in reaches the library's own argument
    # checks (a CPU input is refused) instead of tracing into the launches
    import pytest
    import _tklib as tk

    cfg = StackConfig(1, 8, 128, 4, 128, 1, True)
    model = optimized.OptimizedTransformer(cfg)
    compiled = torch.compile(model, backend="eager")
    with pytest.raises(tk.TKError):
        compiled(torch.randn(1, 8, 128))
