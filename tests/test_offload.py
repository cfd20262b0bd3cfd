"""Host <-> device streaming around the calibration passes (g2ptq_b200.utils.offload_utils),
against the semantics of the reference's prefetch_generator / D2HQueue
(utils/offload_utils.py:36-284): the batches yielded, the ambient write-back
queue and its draining."""

import pytest
import torch

from g2ptq_b200.utils import offload_utils as ou


def _host_tensors(n=10, pinned=False):
    g = torch.Generator().manual_seed(0)
    a = torch.randn(n, 6, 8, generator=g).to(torch.bfloat16)
    b = torch.randn(n, 7, generator=g)
    if pinned:
        a, b = a.pin_memory(), b.pin_memory()
    return a, None, b


@pytest.mark.parametrize("use_prefetch", [False, True])
@pytest.mark.parametrize("bsz", [1, 3, 10, 16])
def test_prefetch_generator_batches_on_cpu(use_prefetch, bsz):
    ts = _host_tensors()
    got = list(ou.prefetch_generator(ts, 10, bsz, "cpu", use_prefetch))
    assert [j for j, _ in got] == list(range(0, 10, bsz))
    for j, batch in got:
        assert len(batch) == 3 and batch[1] is None
        assert torch.equal(batch[0], ts[0][j:j + bsz]) and torch.equal(batch[2], ts[2][j:j + bsz])


def test_ambient_write_back_queue():
    assert isinstance(ou.current_d2h_queue(), ou._ImmediateQueue)
    seen = []
    for _, _ in ou.prefetch_generator((torch.zeros(4),), 4, 2, "cpu"):
        seen.append(ou.current_d2h_queue())
        for _, _ in ou.prefetch_generator((torch.zeros(2),), 2, 1, "cpu"):
            seen.append(ou.current_d2h_queue())
        assert ou.current_d2h_queue() is seen[0]          # the outer loop's queue is back
    assert isinstance(seen[0], ou.D2HQueue) and seen[1] is not seen[0]
    assert isinstance(ou.current_d2h_queue(), ou._ImmediateQueue)


def test_write_back_without_a_device_copies_at_once():
    q = ou.D2HQueue()
    dst, src = torch.zeros(5), torch.arange(5.0)
    q.copy_(dst, src)
    assert torch.equal(dst, src) and not q._done
    h = ou.empty_pinned_like(torch.zeros(3, 2, dtype=torch.int8))
    assert h.shape == (3, 2) and h.dtype == torch.int8
    assert h.is_pinned() == torch.cuda.is_available()


@pytest.mark.gpu
@pytest.mark.parametrize("use_prefetch", [False, True])
def test_prefetch_and_write_back_on_gpu(use_prefetch):
    """Batches arrive equal to the host slices while the next ones copy; each
    batch's result written back through the ambient queue has landed in
    pinned host memory when the loop ends."""
    ts = _host_tensors(n=37, pinned=True)
    out = ou.empty_pinned_like(torch.empty(37, 7))
    assert out.is_pinned()
    out.zero_()
    n = 0
    for j, (a, none, b) in ou.prefetch_generator(ts, 37, 4, "cuda", use_prefetch, depth=3):
        assert a.is_cuda and none is None and b.is_cuda
        assert torch.equal(a.cpu(), ts[0][j:j + 4])
        y = b * 2.0 + a.float().sum(dim=(1, 2))[:, None]   # some work on the consumer stream
        ou.current_d2h_queue().copy_(out[j:j + y.shape[0]], y)
        n += 1
    assert n == 10
    want = ts[2] * 2.0 + ts[0].float().sum(dim=(1, 2))[:, None]
    torch.testing.assert_close(out, want)
