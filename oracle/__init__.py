"""CPU oracle for the fused dynamic causal convolution and the fused source conv.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped library imports this package:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker or as
the timed CPU baseline, never as the thing measured on the GPU.

The functions restate, in numpy, the reference's PyTorch formulas:

* ``fdc``  -- ``torch_reference_materialized_chunk`` and its autograd backward
  (adjfangjiawei/DUDyConv ``test_fused_dynamic_conv_against_reference.py:91-189``).
* ``fscm`` -- ``torch_reference_source_conv_mixed_chunk`` and its autograd
  backward (``test_fused_source_conv_mixed.py:111-255``).

Parity is pinned by ``tests/golden/*.npz``: fixtures produced by importing the
reference's own Python formulas in the build container (script committed as
``tests/golden/make_golden.py``) and checked against this oracle by
``tests/test_oracle_golden.py``.
"""

from .fdc import fdc_forward, fdc_backward, fdc_forward_backward_fp32  # noqa: F401
from .fscm import fscm_forward, fscm_backward  # noqa: F401
