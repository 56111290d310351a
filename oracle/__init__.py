"""CPU oracle for the Transformer layer-stack forward.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or the timed CPU baseline -- never as the thing measured on
the GPU or shipped.

The oracle restates, in fp32 torch on the CPU, the organisers' harness
``src/torch_transformer_benchmark.py`` of danielfodgaard/transformer-kernel:
the model (``BaselineTransformer``), its default weight initialisation, the
seeded input generator and the element-wise acceptance rule. It is pinned
against outputs of the unmodified reference harness, imported in the build
container, stored as fixtures under ``tests/golden/`` together with the
script that generated them.
"""

from .baseline import (  # noqa: F401
    StackConfig,
    AccuracyResult,
    attention_reference,
    chunked_forward,
    compare_outputs,
    generate_random_case,
    init_params,
    layer_norm_reference,
    stack_forward,
    stack_forward_rows,
)
