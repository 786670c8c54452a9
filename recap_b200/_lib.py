"""ctypes binding of librecap_b200.so (the C ABI of include/recap_b200.h).

The library is loaded once.  There is no fallback: if it cannot be loaded, every entry
point raises.  Return codes are mapped onto the reference's exception types: shape and
argument errors raise ``ValueError``, launch failures ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "librecap_b200.so"

ABI_VERSION = 8  # RECAP_B200_ABI_VERSION of include/recap_b200.h

RECAP_OK = 0
RECAP_ERR_SHAPE = 1
RECAP_ERR_LAUNCH = 2
RECAP_ERR_DEVICE = 3
RECAP_ERR_UNSUPPORTED = 4
RECAP_ERR_SCRATCH_LIMIT = 5

STATUS_NAMES = {
    101: "TMA wait timed out",
    102: "MMA wait timed out",
    103: "softmax wait timed out",
    104: "producer wait timed out",
    106: "self-test wait timed out (expected from recap_wait_selftest)",
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "recap_abi_version": (_I, []),
    "recap_layout_gather": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                 _P, _I, _P, _P, _P, _P, _P]),
    "recap_layout_gather_ranks": (_I, [_P, _P, _P, _I, _I, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                       _P, _P, _I, _P, _P, _P, _P, _P]),
    "recap_gather_max_rank": (_I, []),
    "recap_cvk_workspace_floats": (_I64, [_I, _I, _I]),
    "recap_value_key_covariance": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "recap_pool_select": (_I, [_P, _P, _I, _I, _I, _I, _F, _I, _I, _P, _P]),
    "recap_partition_overlap": (_I, [_P, _P, _I64, _P, _P]),
    "recap_kernel_block_mask": (_I, [_P, _I, _I, _I, _P, _P]),
    "recap_closure_workspace_floats": (_I64, [_I, _I, _I]),
    "recap_closure_stats": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "recap_basis_prep": (_I, [_P, _I, _I, _P, _P]),
    "recap_coarse_tail": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _F, _I, _P, _P, _P, _P,
                               _P, _P]),
    "recap_block_sparse_fmha": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P]),
    "recap_refresh_attention": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _P]),
    "recap_refresh_attention_ranks": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, _P, _I, _I, _I64, _I64, _P,
                                           _P, _P, _P, _P]),
    "recap_sparse_step_ranks": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I,
                                     _I64, _I64, _P, _P]),
    "recap_peer_alloc": (_I, [_I64, _P]),
    "recap_peer_free": (_I, [_P]),
    "recap_peer_handle_bytes": (_I, []),
    "recap_peer_export": (_I, [_P, _P]),
    "recap_peer_import": (_I, [_P, _P]),
    "recap_peer_close": (_I, [_P]),
    "recap_push_heads": (_I, [_P, _I, _I, _I, _I, _I, _P, _P]),
    "recap_scatter_rows": (_I, [_P, _I, _I, _I, _P, _I, _I, _I64, _I64, _P]),
    "recap_sparse_step": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "recap_refresh_partials": (_I, [_I, _I]),
    "recap_refresh_detail": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P]),
    "recap_refresh_detail_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P]),
    "recap_exp2_check": (_I, [_P, _P, _I, _P]),
    "recap_wait_selftest": (_I, [_P, _I64, _P, _P]),
}

_lib = None
_load_error: Exception | None = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load the shared library (once) and declare its entry points."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    target = Path(path) if path is not None else LIB_PATH
    if not target.exists():
        raise RuntimeError(
            f"{target.name} is not built; run `python -m recap_b200.build` (needs nvcc, sm_100a)"
        )
    lib = ctypes.CDLL(str(target))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.recap_abi_version() != ABI_VERSION:
        raise RuntimeError(
            f"{target.name} has ABI version {lib.recap_abi_version()}, expected {ABI_VERSION}; rebuild it"
        )
    _lib = lib
    return lib


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a tensor (None stays None)."""
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check(rc: int, what: str) -> None:
    if rc == RECAP_OK:
        return
    if rc == RECAP_ERR_SHAPE:
        raise ValueError(f"{what}: invalid shape, stride or alignment")
    if rc == RECAP_ERR_UNSUPPORTED:
        raise ValueError(f"{what}: unsupported configuration")
    if rc == RECAP_ERR_SCRATCH_LIMIT:
        raise ValueError(
            f"{what}: the problem needs more validation scratch than the library's fixed array "
            "holds (banks * ceil(rows / 32) must be <= 131072)"
        )
    if rc == RECAP_ERR_DEVICE:
        raise RuntimeError(
            f"{what}: a kernel gave up a bounded on-chip wait (device timeout); the status word "
            "names the wait (Operator.check_device_status raises with its name)"
        )
    if rc == RECAP_ERR_LAUNCH:
        raise RuntimeError(f"{what}: CUDA launch or API call failed")
    raise RuntimeError(f"{what}: failed with status {rc}")


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    check(rc, name)
