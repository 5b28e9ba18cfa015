"""Named trace scopes for the profiler, off by default and free when off.

    from tempname_5090_b200.utils import tracing
    with tracing.enabled(), torch.profiler.profile(...) as prof:
        trainer.step(batches)
    path, sha = tracing.export(prof, out_dir / "trace_rank0.json")

`scope(name)` wraps `torch.profiler.record_function` only while tracing is
enabled, so the hot path pays one flag test per scope otherwise.  Scopes mark
the model's per-layer forward/backward, the optimizer, and the phases of the
fused operators (GEMM->RS producer and receiver, AG->GEMM).  Device-side
timing of the fused reduce-scatter (per-tile completion stamps) is separate:
`GemmRS.profile_call`.  Follows the stage/lane scopes and the hashed chrome
trace of TempName-5090 python/flux_5090/runtime.py:176-227 and worker.py:293-300.
"""
from __future__ import annotations

import contextlib
import hashlib
from pathlib import Path

_ON = [False]


def is_enabled() -> bool:
    return _ON[0]


@contextlib.contextmanager
def enabled(on: bool = True):
    """Turn scopes on inside the block (restores the previous state)."""
    prev = _ON[0]
    _ON[0] = on
    try:
        yield
    finally:
        _ON[0] = prev


def scope(name: str):
    if not _ON[0]:
        return contextlib.nullcontext()
    import torch
    return torch.profiler.record_function(name)


def export(prof, path) -> tuple[str, str]:
    """Write a chrome trace; return (path, sha256 of its bytes)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    prof.export_chrome_trace(str(path))
    return str(path), hashlib.sha256(path.read_bytes()).hexdigest()
