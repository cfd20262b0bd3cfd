"""Host <-> device streaming around the calibration passes, a drop-in for the
transport half of utils/offload_utils.py of the reference (:36-287):
``empty_pinned_like``, ``D2HQueue``, ``current_d2h_queue`` and
``prefetch_generator``.

``prefetch_generator`` yields the same ``(j, batch)`` tuples as the
reference's (slices ``[j:j+bsz]`` of each host tensor moved to the device,
``None`` passed through).  With ``use_prefetch`` the copies are issued from
the calling thread on a per-device copy stream, ``depth`` batches ahead
(the reference runs one batch ahead from a worker thread); each batch is
handed over behind an event, and its tensors are recorded on the consumer
stream so the caching allocator does not recycle them while in use.  From
pinned host memory the copies run asynchronously; from pageable memory the
driver stages them, as it does for the reference.

While a loop runs, a ``D2HQueue`` is the ambient write-back queue
(``current_d2h_queue``): device-to-host copies into pinned memory run on a
copy stream behind the producing stream, with a bounded number in flight,
and the queue is drained when the loop ends; outside a loop the ambient
queue copies synchronously.
"""

import collections
import contextlib

import torch


def empty_pinned_like(t):
    """Host tensor of ``t``'s shape and dtype, page-locked when CUDA is present
    (offload_utils.py:36-45), the destination an asynchronous copy needs."""
    return torch.empty(t.shape, dtype=t.dtype, device="cpu",
                       pin_memory=torch.cuda.is_available())


_COPY_STREAMS = {}


def _copy_stream(device_index, direction):
    """One copy stream per device and direction ("h2d" / "d2h"): a write-back
    waits for the compute that produced its source, and on a shared stream
    the prefetch copies queued after it would wait too."""
    key = (device_index, direction)
    s = _COPY_STREAMS.get(key)
    if s is None:
        s = torch.cuda.Stream(device=torch.device("cuda", device_index))
        _COPY_STREAMS[key] = s
    return s


class D2HQueue:
    """Device-to-host write-back overlapped with the following compute
    (offload_utils.py:48-121).  ``copy_(dst, src)`` is asynchronous when ``src``
    is a contiguous CUDA tensor and ``dst`` contiguous pinned host memory, and a
    plain blocking copy otherwise; at most ``max_inflight`` asynchronous copies
    are outstanding (each keeps its source alive); ``wait()`` blocks until all
    have landed."""

    def __init__(self, max_inflight=2):
        self.max_inflight = max_inflight
        self._done = collections.deque()

    @staticmethod
    def _async_ok(dst, src):
        return (src.is_cuda and dst.device.type == "cpu" and dst.is_pinned()
                and dst.is_contiguous() and src.is_contiguous())

    def copy_(self, dst, src):
        if not self._async_ok(dst, src):
            dst.copy_(src)
            return
        dev = src.device.index
        stream = _copy_stream(dev, "d2h")
        stream.wait_stream(torch.cuda.current_stream(dev))  # behind the producer of src
        with torch.cuda.stream(stream):
            dst.copy_(src, non_blocking=True)
            src.record_stream(stream)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._done.append(ev)
        while len(self._done) > self.max_inflight:
            self._done.popleft().synchronize()

    def wait(self):
        while self._done:
            self._done.popleft().synchronize()


class _ImmediateQueue:
    """Ambient queue outside a prefetch loop: copies at once."""

    def copy_(self, dst, src):
        dst.copy_(src)

    def wait(self):
        pass


_IMMEDIATE = _ImmediateQueue()
_active_queue = None


def current_d2h_queue():
    """The write-back queue of the enclosing ``prefetch_generator`` loop, or an
    immediate one outside any loop (offload_utils.py:134-140)."""
    return _active_queue if _active_queue is not None else _IMMEDIATE


@contextlib.contextmanager
def _installed_d2h_queue():
    """A fresh ambient ``D2HQueue`` for the duration of a loop, drained on exit;
    a queue left behind by an abandoned loop is drained first
    (offload_utils.py:147-170)."""
    global _active_queue
    if _active_queue is not None:
        _active_queue.wait()
    previous = _active_queue
    q = D2HQueue()
    _active_queue = q
    try:
        yield q
    finally:
        q.wait()
        _active_queue = previous


def _slice_to(t, j, bsz, device):
    if t is None:
        return None
    return t[j:j + bsz].to(device, non_blocking=True)


def prefetch_generator(tensors, num_samples, bsz, onload_device, use_prefetch=False, depth=2):
    """Yield ``(j, batch)`` for ``j = 0, bsz, 2 bsz, ... < num_samples`` with
    ``batch[i] = tensors[i][j:j+bsz]`` on ``onload_device`` (``None`` entries
    stay ``None``), the reference's prefetch_generator (offload_utils.py:203-284).
    With ``use_prefetch`` and a CUDA ``onload_device`` the next ``depth``
    batches are already copying on a side stream while a batch is consumed."""
    device = torch.device(onload_device)
    starts = list(range(0, num_samples, bsz))
    with _installed_d2h_queue():
        if not (use_prefetch and device.type == "cuda"):
            for j in starts:
                yield j, tuple(_slice_to(t, j, bsz, device) for t in tensors)
            return
        dev_index = device.index if device.index is not None else torch.cuda.current_device()
        copy = _copy_stream(dev_index, "h2d")
        consumer = torch.cuda.current_stream(dev_index)
        pending = collections.deque()

        def issue(j):
            # the batch is allocated on the copy stream and recorded on the
            # consumer's, so its memory returns to the pool only after the
            # consumer's use of it: no wait on the consumer here
            with torch.cuda.stream(copy):
                batch = tuple(_slice_to(t, j, bsz, device) for t in tensors)
                for b in batch:
                    if b is not None:
                        b.record_stream(consumer)
            ev = torch.cuda.Event()
            ev.record(copy)
            pending.append((j, batch, ev))

        nxt = 0
        for _ in starts:
            while nxt < len(starts) and len(pending) <= depth:
                issue(starts[nxt])
                nxt += 1
            j, batch, ev = pending.popleft()
            consumer.wait_event(ev)
            yield j, batch
