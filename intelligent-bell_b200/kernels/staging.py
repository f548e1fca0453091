"""Small host-side call arguments (page tables, lengths, shifts, offsets) moved to the GPU.

A copy from pageable host memory is synchronous: the calling thread waits until the work
already queued on the stream has drained, so a call that takes its lengths or shifts as a
Python list would serialise the host with the GPU.  Here every host-side argument of one
call is packed into one pinned buffer (from torch's caching host allocator) and sent with a
single asynchronous copy on the current stream; the kernel launched after it on the same
stream reads the device copy.  The pinned block is recycled only after the copy completes.
"""

from __future__ import annotations

import torch

_ALIGN = 16  # bytes; every array starts on a 16-byte boundary of the staged buffer


def host_array(x, dtype: torch.dtype) -> torch.Tensor:
    """``x`` (list, number, numpy array or tensor) as a contiguous tensor of ``dtype``.

    Device tensors stay on their device; everything else becomes a host tensor.
    """
    t = x if isinstance(x, torch.Tensor) else torch.as_tensor(x)
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def to_device(tensors: list[torch.Tensor], device: torch.device) -> list[torch.Tensor]:
    """Device versions of ``tensors`` (contiguous, already of their final dtype).

    Tensors on ``device`` are returned as they are, tensors on another GPU are copied, and
    all host tensors travel together in one asynchronous pinned-memory copy.
    """
    out = list(tensors)
    host = [i for i, t in enumerate(tensors) if not t.is_cuda]
    for i, t in enumerate(tensors):
        if t.is_cuda and t.device != device:
            out[i] = t.to(device)
    if not host:
        return out
    nbytes = [tensors[i].numel() * tensors[i].element_size() for i in host]
    spans = [(n + _ALIGN - 1) // _ALIGN * _ALIGN for n in nbytes]
    buf = torch.empty(max(sum(spans), _ALIGN), dtype=torch.uint8, pin_memory=True)
    off = 0
    for i, n, span in zip(host, nbytes, spans):
        if n:
            buf[off:off + n].copy_(tensors[i].reshape(-1).view(torch.uint8))
        off += span
    with torch.cuda.device(device):
        dev_buf = buf.to(device, non_blocking=True)
    off = 0
    for i, n, span in zip(host, nbytes, spans):
        t = tensors[i]
        out[i] = dev_buf[off:off + n].view(t.dtype).view(t.shape)
        off += span
    return out
