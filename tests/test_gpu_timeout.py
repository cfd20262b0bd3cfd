"""Bounded pipeline waits of the tensor-core kernels (GPU).

Every mbarrier wait in the tcgen05 kernels gives up after a bound that
``g2q_set_wait_limit`` sets.  With a bound far below the latency of a TMA
load, the first wait on a load runs out: the kernel must record
G2Q_ERR_TIMEOUT in the call's status word, let the loads it issued land,
free its TMEM and return, so that the CUDA context stays usable and the next
call with the default bound is correct.  The case is a single-CTA tile shape
(C = 256 < 512 columns), whose producer arms every barrier it waits on.
"""

import pytest
import torch

from g2ptq_b200 import _lib, ops

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _gram_case(seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    X = torch.randn(4096, 256, device=DEV, generator=g).to(torch.bfloat16)
    return X


def test_wait_that_runs_out_reports_timeout_and_context_survives():
    lib = _lib.load()
    X = _gram_case(3)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    D = torch.zeros(256, 256, device=DEV)
    prev = lib.g2q_set_wait_limit(64)  # far below a TMA load's latency
    try:
        ops.gram_update(D, X, precision=1, status=status)
        torch.cuda.synchronize()
    finally:
        lib.g2q_set_wait_limit(prev)
    assert int(status.item()) == _lib.G2Q_ERR_TIMEOUT

    # the context is intact: the same call with the default bound is correct
    status.zero_()
    D2 = torch.zeros(256, 256, device=DEV)
    ops.gram_update(D2, X, precision=1, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = X.double().T @ X.double()
    err = float((D2.double() - ref).norm() / ref.norm())
    assert err < 1e-5, err


def test_timeout_in_fasterquant_raises():
    """A timed-out fold leaves the device status word set; the next
    fasterquant reads it with its other status words and raises."""
    from g2ptq_b200.gptq_utils import gptq_utils
    from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers
    from g2ptq_b200.utils.quant_utils import WeightQuantizer
    lib = _lib.load()
    lin = torch.nn.Linear(256, 128, bias=False, device=DEV)
    obj = gptq_utils.GPTQ([lin])
    q = WeightQuantizer()
    q.configure(4, perchannel=True, sym=True)
    obj.quantizer = make_group_quantizers(q, 256, 128)
    obj.add_batch(0, _gram_case(4)[None], None)
    word = ops.device_status(DEV)
    word.zero_()
    prev = lib.g2q_set_wait_limit(64)
    try:
        obj._flush_all()  # the Gram fold runs now, with the short bound
        torch.cuda.synchronize()
    finally:
        lib.g2q_set_wait_limit(prev)
    try:
        assert int(word.item()) == _lib.G2Q_ERR_TIMEOUT
        with pytest.raises(RuntimeError, match="timed out"):
            obj.fasterquant(groupsize=128)
    finally:
        word.zero_()
        torch.cuda.synchronize()
