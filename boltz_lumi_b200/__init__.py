"""B200-native (sm_100a) kernels for Boltz-2's pair-representation hot path.

Drop-in for the module API of upstream Boltz 2.2.1:

* :func:`boltz_lumi_b200.adapters.install` rebinds the forwards of a loaded
  Boltz-2 model (TriangleAttention / EndingNode, TriangleMultiplication
  Outgoing / Incoming, the pair Transition, diffusion AdaLN /
  ConditionedTransitionBlock);
* :mod:`boltz_lumi_b200.layers` holds standalone modules with the upstream
  constructors and parameter names;
* ``python -m boltz_lumi_b200 predict ...`` wraps the Boltz CLI.

All compute runs in ``libboltz_b200.so`` (C ABI: ``include/boltz_b200.h``).
"""

SUPPORTED_BOLTZ_VERSION = "2.2.1"
__version__ = "0.1.0"
