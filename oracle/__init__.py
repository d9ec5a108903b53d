"""CPU oracle for the Boltz-2 pair-representation hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may use it, and only as the checker.

The oracle restates, in plain PyTorch on the CPU, the eager ``--no_kernels``
semantics of upstream Boltz 2.2.1 (the reference's pip dependency,
``requirements.txt:1`` of lauritsf/boltz-lumi, commit cb04aec; not vendored,
not installable here) under bf16 autocast, including every bf16 rounding point
the reference's kernels preserve.  Parity status:

* kernel-level formulas (ordered bias softmax, SiLU-mul, sigmoid gate,
  diffusion epilogues) are pinned against the reference tests' own reference
  expressions (``tests/golden/make_golden.py`` evaluates them and the fixtures
  under ``tests/golden/`` hold the results);
* module-level semantics (TriangleAttention, TriangleMultiplication,
  Transition, AdaLN, ConditionedTransitionBlock, the Pairformer block) are
  restated from the reference's adapter code and the published AF3/Boltz
  algorithms: **parity unpinned** against upstream itself, because upstream
  cannot run in this environment.
"""

from .numerics import GATE, GATED_SWIGLU, MODULATION, bf16_round, diffusion_epilogue, linear_bf16, sigmoid_bf16  # noqa: F401
from .modules import (  # noqa: F401
    AdaLN,
    Attention,
    AttentionPairBias,
    ConditionedTransitionBlock,
    LayerNorm,
    PairformerLayer,
    Transition,
    TriangleAttention,
    TriangleAttentionEndingNode,
    TriangleMultiplicationIncoming,
    TriangleMultiplicationOutgoing,
    ordered_bias_softmax,
    randomize,
)
