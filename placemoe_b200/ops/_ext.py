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


_P2P_STATUS: dict = {}

# identifiers of the wait that gave up first (status word 1, see csrc/kernels/peer.cuh)
_WAIT_NAMES = {1: "p2p barrier", 2: "grid barrier", 3: "dispatch count exchange", 4: "dispatch rows",
               5: "combine partial sums", 6: "backward scatter", 7: "index check (debug build)",
               8: "sequence-parallel exchange"}
_ERROR_NAMES = {1: "mbarrier wait timed out", 2: "peer wait timed out", 3: "bounds check failed", 4: "bad arguments"}


def p2p_status(device) -> "torch.Tensor":
    """Sticky status block (int32[4]) shared by every peer-memory kernel on ``device``.

    Word 0 is the first error code (0 = ok), word 1 the wait that gave up, word 2
    the largest received row count seen.  Once word 0 is set, every later peer
    wait returns at once, so a missing peer costs one time budget per process.
    """
    import torch

    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    st = _P2P_STATUS.get(dev)
    if st is None:
        st = torch.zeros(4, dtype=torch.int32, device=dev)
        _P2P_STATUS[dev] = st
    return st


def device_error(reset: bool = True) -> int:
    """Error word written by bounded device waits / checks (0 = no error)."""
    code = int(kernels().device_error(reset))
    for st in _P2P_STATUS.values():
        v = int(st[0].item())
        if v and not code:
            code = v
        if reset and v:
            st[:2].zero_()
    return code


def check_device_error() -> None:
    """Raise if any kernel recorded an error since the last check (one small device read per source)."""
    where = ""
    for st in _P2P_STATUS.values():
        w = st[:2].tolist()
        if w[0]:
            where = f" (first failed wait: {_WAIT_NAMES.get(w[1], w[1])})"
            break
    code = device_error(reset=True)
    if code:
        raise RuntimeError(f"placemoe_b200 kernel reported error {code}: {_ERROR_NAMES.get(code, 'unknown')}{where}")
