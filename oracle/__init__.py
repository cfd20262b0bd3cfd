"""CPU oracle for the G2PTQ per-layer quantization hot path (TEST INFRASTRUCTURE).

This package is a numpy float32 restatement of the reference's torch code for
the quantizer objects (``gptq_utils/{gptq,g2ptq,gptaq,gptq_guided}_utils.py``,
``gptq_utils/common_utils.py``, ``utils/quant_utils.py``,
``utils/compressed_tensors_utils.py``).  Every function cites the reference
``file:line`` it follows.

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` -- and there only
as the checker or the timed CPU baseline.  The product path
(``g2ptq_b200``) never imports it and has no CPU fallback.

Pinning: the restatement is checked against golden fixtures produced by
running the reference itself on CPU (``tests/golden/make_golden.py`` imports
the reference's own ``gptq_utils`` with stubs for its missing third-party
modules and writes ``tests/golden/*.npz``); ``tests/test_oracle_golden.py``
holds the comparison.
"""

from . import quant, hessian, linalg, compensation, fasterquant, export, partition, refresh  # noqa: F401,E501
