"""Access to the compiled sm_100a kernel library (``graspo_b200._C``).

The library is built in-tree (``python setup.py build_ext --inplace``).  On a
machine with a GPU the fused path requires it: a missing or stale library is an
error, never a silent fallback to PyTorch.  Each device gets a small int32
error word that kernels set when a bounded wait gives up; ``check_errors``
turns it into an exception at the next host synchronisation point.
"""

from __future__ import annotations

import torch

_C = None
_ERR: dict[int, torch.Tensor] = {}

ERROR_NAMES = {
    1: "TMA tile never arrived (full-barrier timeout)",
    2: "shared-memory stage never released (empty-barrier timeout)",
    3: "accumulator never completed (TMEM full timeout)",
    4: "accumulator never released (TMEM empty timeout)",
    5: "peer GPU never signalled (cross-GPU flag timeout)",
    6: "bad shape",
    7: "index outside its table (kernel-checks build; the access was clamped)",
}


class KernelTimeout(RuntimeError):
    """A kernel's bounded wait expired; the kernel exited without finishing."""


class LaunchCounter:
    """Counts launches of this library's kernels (each entry point launches one).

    Kernels replayed from a CUDA graph are added by the code that replays the
    graph (``add``), since no Python call happens on replay.
    """

    def __init__(self) -> None:
        self.count = 0

    def add(self, n: int) -> None:
        self.count += int(n)

    def reset(self) -> int:
        value, self.count = self.count, 0
        return value


launches = LaunchCounter()


class _Counting:
    def __init__(self, module) -> None:
        self._module = module
        self._cache: dict[str, object] = {}

    def __getattr__(self, name: str):
        fn = self._cache.get(name)
        if fn is None:
            raw = getattr(self._module, name)

            def fn(*args, _raw=raw, **kwargs):
                launches.count += 1
                return _raw(*args, **kwargs)

            self._cache[name] = fn
        return fn


def ext():
    """The loaded extension module; raises if it has not been built."""
    global _C
    if _C is None:
        try:
            from graspo_b200 import _C as module  # type: ignore[attr-defined]
        except ImportError as exc:  # pragma: no cover - depends on the build
            raise RuntimeError(
                "graspo_b200._C (the sm_100a kernel library) is not built; run "
                "`python setup.py build_ext --inplace` in the repository root"
            ) from exc
        _C = _Counting(module)
    return _C


def available() -> bool:
    try:
        ext()
    except RuntimeError:
        return False
    return True


def err_word(device: torch.device | int | None = None) -> torch.Tensor:
    if isinstance(device, torch.device) and device.type == "cpu":
        word = _ERR.get(-1)
        if word is None:
            word = _ERR[-1] = torch.zeros(4, dtype=torch.int32)
        return word
    if device is None:
        device = torch.cuda.current_device()
    index = device if isinstance(device, int) else (device.index if device.index is not None else torch.cuda.current_device())
    word = _ERR.get(index)
    if word is None:
        word = torch.zeros(4, dtype=torch.int32, device=f"cuda:{index}")
        _ERR[index] = word
    return word


def check_errors(device: torch.device | int | None = None) -> None:
    """Raise ``KernelTimeout`` if any kernel on ``device`` reported a failure."""
    word = err_word(device)
    code = int(word[0].item())
    if code:
        word.zero_()
        raise KernelTimeout(f"kernel error {code}: {ERROR_NAMES.get(code, 'unknown')}")
