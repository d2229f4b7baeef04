"""Activation offload: tensors saved for the backward move to pinned host memory.

Inside ``ActivationOffload()``, every CUDA tensor that autograd saves for the
backward and that has at least ``min_bytes`` bytes is copied to pinned host
memory on a side stream (ordered after the producing work on the current
stream) and the device copy is released; the backward copies it back on its
first use.  Small tensors and parameters stay on the device.  This trades
PCIe traffic for HBM, for runs whose activations do not fit; it does not
change any result.

Reference parity: activation CPU offload of veomni/distributed/offloading.py:26-199.
"""

from __future__ import annotations

import torch


class _Offloaded:
    __slots__ = ("host", "event", "device", "dtype", "shape")

    def __init__(self, t: torch.Tensor, stream: torch.cuda.Stream):
        self.device, self.dtype, self.shape = t.device, t.dtype, t.shape
        self.host = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=True)
        cur = torch.cuda.current_stream(t.device)
        stream.wait_stream(cur)
        with torch.cuda.stream(stream):
            self.host.copy_(t, non_blocking=True)
            t.record_stream(stream)  # the device copy stays alive until the transfer ran
            self.event = torch.cuda.Event()
            self.event.record(stream)

    def restore(self) -> torch.Tensor:
        self.event.synchronize()  # the host copy is complete
        return self.host.to(self.device, non_blocking=True)


class ActivationOffload:
    """Context manager; ``min_bytes`` = smallest saved tensor worth moving (default 1 MiB)."""

    def __init__(self, min_bytes: int = 1 << 20, enabled: bool = True):
        self.min_bytes = min_bytes
        self.enabled = enabled
        self.stream = None
        self.offloaded_bytes = 0
        self._hooks = None

    def _pack(self, t: torch.Tensor):
        if (not t.is_cuda or t.numel() * t.element_size() < self.min_bytes or isinstance(t, torch.nn.Parameter)
                or t.requires_grad and t.grad_fn is None):
            return t
        if self.stream is None:
            self.stream = torch.cuda.Stream(device=t.device)
        self.offloaded_bytes += t.numel() * t.element_size()
        return _Offloaded(t, self.stream)

    @staticmethod
    def _unpack(x):
        return x.restore() if isinstance(x, _Offloaded) else x

    def __enter__(self):
        if self.enabled:
            self._hooks = torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack)
            self._hooks.__enter__()
        return self

    def __exit__(self, *exc):
        if self._hooks is not None:
            self._hooks.__exit__(*exc)
            self._hooks = None
        return False
