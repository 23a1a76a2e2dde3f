"""Loader for the sm_100a extension ``granite_switch_b200._C``.

The extension is built in place (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``). On a CUDA device every op in
:mod:`granite_switch_b200.ops` calls it; when it is missing there, the op
raises instead of silently running a slower PyTorch path.
"""
from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_C = None
_err_buffers: dict[int, torch.Tensor] = {}

# Bits of the device error word (csrc/common.cuh, enum ErrorBits).
ERR_GEMM_WAIT = 1 << 0
ERR_ATTN_WAIT = 1 << 1
ERR_PEER_WAIT = 1 << 2
ERR_BAD_SHAPE = 1 << 3
ERR_SHRINK_WAIT = 1 << 4


class NativeExtensionMissing(RuntimeError):
    pass


_REPLAYED = 0  # kernels run by CUDA-graph replays (the extension counts host launches)


def launch_count() -> int:
    """Kernels this extension launched so far: every launch it issued from the host
    (counted in the extension, one per launch configuration, split-K reduces and
    split-KV merges included) plus the kernels of CUDA-graph replays reported
    through :func:`add_launches`. 0 before the extension is loaded."""
    return (int(_C.kernel_launches()) if _C is not None else 0) + _REPLAYED


def add_launches(n: int) -> None:
    """Account for ``n`` kernel launches issued by a CUDA-graph replay."""
    global _REPLAYED
    _REPLAYED += n


def native():
    """Return the loaded extension, importing it on first use."""
    global _C
    if _C is None:
        with _lock:
            if _C is None:
                try:
                    from . import _C as mod  # type: ignore[attr-defined]
                except ImportError as e:  # pragma: no cover - depends on build state
                    raise NativeExtensionMissing(
                        "granite_switch_b200._C is not built; run "
                        "`python setup.py build_ext --inplace` in the repository root"
                    ) from e
                _C = mod
    return _C


def available() -> bool:
    try:
        native()
        return True
    except NativeExtensionMissing:
        return False


def err_buffer(device: torch.device) -> torch.Tensor:
    """Per-device int32[4] word that bounded device waits report into.

    Allocated on first use; call once per device before CUDA-graph capture.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _err_buffers.get(idx)
    if buf is None:
        buf = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_buffers[idx] = buf
    return buf


# Sites of bad-index reports (csrc/common.cuh, enum BadIndexSite): err[1] holds the
# first report's site, err[2] its index.
BAD_INDEX_SITES = {1: "embedding token id", 2: "rotary position", 3: "KV slot", 4: "attention page id",
                   5: "tcgen05 attention page id"}


def read_errors(device: torch.device, clear: bool = True) -> int:
    """Synchronise and return (optionally clearing) the device error word."""
    return read_error_detail(device, clear)[0]


def read_error_detail(device: torch.device, clear: bool = True) -> tuple[int, str | None, int | None]:
    """``(error word, site of the first bad index or None, that index)``."""
    buf = err_buffer(device)
    w, site, idx = (int(v) for v in buf[:3].tolist())
    if clear and (w or site):
        buf.zero_()
    if not site:
        return w, None, None
    return w, site_name(site), idx


class DeviceError(RuntimeError):
    """Kernels of a step reported a bounded wait that ran out or a bad index.

    ``word`` is the device error word (``ERR_*`` bits); ``site`` / ``index`` the
    first bad index reported, if any. The outputs of that step are not to be
    trusted: the engine aborts the requests the step carried.
    """

    def __init__(self, word: int, site: str | None = None, index: int | None = None):
        self.word, self.site, self.index = int(word), site, index
        super().__init__(describe_error(self.word, site, index))


_ERR_NAMES = ((ERR_GEMM_WAIT, "gemm-wait-timeout"), (ERR_ATTN_WAIT, "attention-wait-timeout"),
              (ERR_PEER_WAIT, "peer-wait-timeout"), (ERR_BAD_SHAPE, "bad-shape"),
              (ERR_SHRINK_WAIT, "shrink-wait-timeout"))


def describe_error(word: int, site: str | None = None, index: int | None = None) -> str:
    names = [name for bit, name in _ERR_NAMES if word & bit] or ["unknown"]
    where = f"; first bad index: {site} = {index}" if site else ""
    return f"device kernels reported errors: {', '.join(names)} (0x{word:x}){where}"


def site_name(code: int) -> str | None:
    """Name of a bad-index site code (``err[1]``), or None for 0."""
    return BAD_INDEX_SITES.get(code, f"site {code}") if code else None


def check_errors(device: torch.device) -> None:
    val, site, idx = read_error_detail(device)
    if val:
        raise DeviceError(val, site, idx)
