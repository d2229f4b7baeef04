"""Access to the compiled sm_100a kernel module.

The CUDA path of every op in :mod:`placemoe_b200.ops` goes through
:func:`kernels`.  If the extension is missing on a machine with a GPU the
import error propagates: there is no silent eager fallback for CUDA tensors.
CPU tensors take the PyTorch reference path of each op (used by the gloo
multi-process tests and as the numerical oracle).
"""

from __future__ import annotations

import functools

from .. import _build


# kernel launches issued by one call of each entry point (for launch accounting)
LAUNCHES_PER_CALL = {"moe_plan": 4, "attn_bwd": 3}


class _CountingModule:
    """Proxy over the extension module that counts entry-point calls (launch accounting)."""

    def __init__(self, mod):
        self._mod = mod
        self.calls: dict = {}
        self.counting = False

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def wrapped(*args, **kwargs):
            if self.counting:
                self.calls[name] = self.calls.get(name, 0) + 1
            return fn(*args, **kwargs)

        return wrapped

    def launches(self) -> int:
        return sum(LAUNCHES_PER_CALL.get(k, 1) * v for k, v in self.calls.items() if k != "device_error")

    def reset(self):
        self.calls = {}


@functools.lru_cache(maxsize=1)
def kernels():
    return _CountingModule(_build.load_kernels())


def available() -> bool:
    try:
        kernels()
        return True
    except ImportError:
        return False


def device_error(reset: bool = True) -> int:
    """Error word written by bounded device waits / checks (0 = no error)."""
    return int(kernels().device_error(reset))


def check_device_error() -> None:
    code = device_error(reset=True)
    if code:
        names = {1: "mbarrier wait timed out", 2: "peer wait timed out", 3: "bounds check failed", 4: "bad arguments"}
        raise RuntimeError(f"placemoe_b200 kernel reported error {code}: {names.get(code, 'unknown')}")
