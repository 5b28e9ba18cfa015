"""Loader for the in-tree native extension (tempname_5090_b200._C).

On a machine with CUDA the extension is mandatory: `lib()` raises if it cannot
be imported, so no CUDA code path silently runs anything else.  CPU-only hosts
(unit tests) never call it.
"""
from __future__ import annotations

import threading
import weakref

_LOCK = threading.Lock()
# Live fused operators and exchange workspaces (objects with a `failed`
# attribute): a device-side bounded-wait failure poisons all of them.
_OPERATORS: "weakref.WeakSet" = weakref.WeakSet()
_LIB = None
_ERROR: Exception | None = None
_STATUS: dict = {}
_LAUNCHES = [0]

STATUS_MESSAGES = {
    1: "GEMM producer timed out waiting for a free shared-memory stage",
    2: "GEMM MMA warp timed out waiting for a loaded stage",
    3: "GEMM MMA warp timed out waiting for the epilogue to drain TMEM",
    4: "GEMM epilogue timed out waiting for an accumulator",
    5: "a cross-GPU readiness flag never arrived (peer stalled or failed)",
    6: "abort drain of in-flight copies timed out",
    7: "AG->GEMM: a gathered row chunk never arrived",
    8: "bad kernel argument",
}


def lib():
    """Return the native module; raise if it is unavailable."""
    global _LIB, _ERROR
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            try:
                import torch  # noqa: F401  (loads the libraries the extension links against)
                from . import _C  # type: ignore
                _LIB = _C
            except Exception as exc:  # pragma: no cover - depends on build state
                _ERROR = exc
                raise RuntimeError(
                    "tempname_5090_b200 native extension is not built or failed to load; "
                    "run `python setup.py build_ext --inplace` (sm_100a). "
                    f"Import error: {exc}") from exc
    return _LIB


def available() -> bool:
    try:
        lib()
        return True
    except RuntimeError:
        return False


def status_tensor(device):
    """Per-device int32 status word shared by all kernels' bounded waits."""
    import torch
    device = torch.device(device)
    if device.type == "cpu":  # host-logic tests: a stand-in word nothing writes
        t = _STATUS.get("cpu")
        if t is None:
            t = _STATUS["cpu"] = torch.zeros(4, dtype=torch.int32)
        return t
    index = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(index)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", index))
        _STATUS[index] = t
    return t


def register_operator(op) -> None:
    """Track a fused operator or exchange workspace for device-failure poisoning."""
    _OPERATORS.add(op)


def poison_operators() -> int:
    """Mark every live fused operator and workspace failed; returns how many.
    After a bounded wait gave up, a peer's late pushes or pulls of that epoch
    may still be in flight, and cumulative counters are out of step: these
    objects must be rebuilt, not called again."""
    n = 0
    for op in list(_OPERATORS):
        op.failed = True
        n += 1
    return n


def check_status(device=None, clear: bool = True) -> None:
    """Synchronise and raise if any kernel recorded a bounded-wait failure;
    every live fused operator and workspace is poisoned first."""
    import torch
    index = torch.cuda.current_device() if device is None else torch.device(device).index
    t = _STATUS.get(index)
    if t is None:
        return
    code = int(t[0].item())
    if code:
        poisoned = poison_operators()
        if clear:
            t.zero_()
        raise RuntimeError(f"device status {code}: {STATUS_MESSAGES.get(code, 'unknown')} "
                           f"({poisoned} fused operators/workspaces poisoned: rebuild them)")


def count_launch(n: int = 1) -> None:
    _LAUNCHES[0] += n


def launches() -> int:
    return _LAUNCHES[0]
