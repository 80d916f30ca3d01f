"""ctypes binding of ``libsparsevox.so``, the sm_100a CUDA library behind this package.

There is no CPU fallback: if the shared library is missing, or a tensor is not on a CUDA
device, the calls raise. Arrays cross the boundary as raw device pointers taken from torch
tensors (other frameworks' arrays are accepted through DLPack, see :func:`as_tensor`).
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libsparsevox.so")

# sv_status
SV_OK = 0
SV_ERR_INVALID_ARGUMENT = 1
SV_ERR_BAD_SHAPE = 2
SV_ERR_BAD_DTYPE = 3
SV_ERR_TABLE_FULL = 4
SV_ERR_CUDA = 5
SV_ERR_UNSUPPORTED = 6
SV_ERR_WORKSPACE = 7

# sv_weight_layout / sv_conv_algo
SV_WEIGHT_KIO = 0
SV_WEIGHT_OKI = 1
SV_CONV_AUTO = 0
SV_CONV_SIMT = 1
SV_CONV_TCGEN05 = 2
SV_CONV_TCGEN05_DEDUP = 3  # Python-level choice: sv_conv_dd_plan + sv_conv3d_forward_dd

# device status bits
SV_DEVICE_TABLE_FULL = 0x1
SV_DEVICE_BAD_INDEX = 0x2
SV_DEVICE_WAIT_TIMEOUT = 0x4

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_SZ = ctypes.c_size_t

_SIGNATURES = {
    "sv_last_error": (ctypes.c_char_p, []),
    "sv_abi_version": (_I32, []),
    "sv_kmap_table_slots": (_I64, [_I64]),
    "sv_kmap_workspace_bytes": (_SZ, [_I64]),
    "sv_kmap_build": (_I32, [_P, _I64, _P, _P, _P, _I64, _P, _SZ, _P, _P]),
    "sv_kmap_build_static": (_I32, [_P, _I64, _P, _P, _P, _P, _P]),
    "sv_coords_bounds": (_I32, [_P, _I64, _P, _P, _SZ, _P]),
    "sv_kmap_grid_workspace_bytes": (_SZ, [_P]),
    "sv_kmap_build_grid": (_I32, [_P, _I64, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "sv_kmap_auto_workspace_bytes": (_SZ, [_I64]),
    "sv_kmap_build_auto": (_I32, [_P, _I64, _P, _P, _P, _P, _SZ, _P, _P]),
    "sv_conv_plan_tiles": (_I64, [_I64]),
    "sv_conv_plan_workspace_bytes": (_SZ, [_I64]),
    "sv_conv_plan": (_I32, [_P, _I64, _I32, _P, _P, _P, _SZ, _P]),
    "sv_conv3d_workspace_bytes": (_SZ, [_I64, _I32, _I32, _I32, _I32, _I32, _I32]),
    "sv_conv3d_forward": (
        _I32,
        [_P, _I64, _I32, _P, _I32, _P, _P, _P, _I32, _P, _I32, _I32, _P, _I32, _P, _SZ, _P, _P],
    ),
    "sv_conv3d_forward_residual": (
        _I32,
        [_P, _I64, _I32, _P, _I32, _P, _P, _P, _I32, _P, _P, _I32, _I32, _P, _I32, _P, _SZ, _P,
         _P],
    ),
    "sv_conv3d_forward_rows": (
        _I32,
        [_P, _I64, _I32, _P, _I32, _P, _I64, _P, _P, _I32, _P, _P, _I32, _I32, _P, _I32, _P,
         _SZ, _P, _P],
    ),
    "sv_conv3d_forward_halo": (
        _I32,
        [_P, _I64, _I32, _P, _I32, _P, _I64, _P, _I32, _P, _I32, _I64, _P, _P, _P, _I32, _I32,
         _P, _P, _SZ, _P, _P],
    ),
    "sv_conv_dd_supported": (_I32, [_I64, _I32, _I32, _I32, _I32]),
    "sv_conv_dd_plan_bytes": (_SZ, [_I64, _I32]),
    "sv_conv_dd_plan_workspace_bytes": (_SZ, [_I64]),
    "sv_conv_dd_plan": (_I32, [_P, _P, _I64, _I32, _I32, _P, _SZ, _P, _SZ, _P, _P]),
    "sv_conv3d_forward_dd": (
        _I32, [_P, _I64, _I32, _P, _I32, _P, _SZ, _P, _P, _P, _I32, _I32, _P, _P, _SZ, _P, _P]
    ),
    "sv_weight_kio_to_oki": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _P]),
    "sv_rownorm": (
        _I32,
        [_P, _I64, _I32, _I32, ctypes.c_float, _P, _P, _P, _P, _I64, _P, _I64, _I32, _P, _P,
         _P],
    ),
    "sv_downsample_workspace_bytes": (_SZ, [_I64]),
    "sv_downsample_coords": (_I32, [_P, _I64, _I32, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sv_downsample_features": (_I32, [_P, _I64, _I32, _I32, _P, _P, _I64, _P, _P]),
    "sv_upsample_features": (_I32, [_P, _I64, _I32, _I32, _P, _I64, _P, _P, _P]),
    "sv_kmap_pairs_workspace_bytes": (_SZ, [_I64, _I32]),
    "sv_kmap_pairs_count": (_I32, [_P, _I64, _I32, _P, _P, _SZ, _P, _P]),
    "sv_kmap_pairs_emit": (_I32, [_P, _I64, _I32, _P, _P, _P, _I64, _P, _SZ, _P, _P]),
    "sv_weight_flip_transpose": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _P]),
    "sv_conv3d_wgrad_workspace_bytes": (_SZ, [_I32, _I32, _I32, _I32, _I32]),
    "sv_conv3d_wgrad": (
        _I32, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _I32, _P, _SZ, _P, _P]
    ),
    "sv_conv3d_dbias_workspace_bytes": (_SZ, [_I64, _I32]),
    "sv_conv3d_dbias": (_I32, [_P, _I64, _I32, _I32, _P, _P, _SZ, _P]),
    "sv_ipc_handle": (_I32, [_P, _P, _P]),
    "sv_ipc_open": (_I32, [_P, _P]),
    "sv_ipc_close": (_I32, [_P]),
    "sv_halo_push": (_I32, [_P, _I64, _I32, _P, _P, _P, _I64, _P, _P, _I32, _P, _P]),
    "sv_halo_signal": (_I32, [_P, _I32, _I64, _P]),
    "sv_halo_wait": (_I32, [_P, _I32, _I64, _P, _P]),
    "sv_occupancy_workspace_bytes": (_SZ, [_P]),
    "sv_occupancy_count": (_I32, [_P, _I32, _P, _P, ctypes.c_double, _P, _P, _SZ, _P]),
    "sv_occupancy_emit": (_I32, [_P, _I32, _P, _P, ctypes.c_double, _P, _I64, _P, _P, _SZ, _P]),
    "sv_subdivide": (_I32, [_P, _I64, _P, _I64, _P, _P, _P]),
    "sv_window_groups_workspace_bytes": (_SZ, [_I64]),
    "sv_window_groups": (_I32, [_P, _I64, _I32, _P, _P, _P, _P, _P, _SZ, _P]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""

    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing; build it with "
                        "`python -m mlx_diffuser_b200.csrc.build` (needs nvcc)"
                    )
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Map an sv_status to the reference's exception types (ValueError for shape/dtype)."""

    if rc == SV_OK:
        return
    msg = load().sv_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if msg else f"{what}: status {rc}"
    if rc in (SV_ERR_BAD_SHAPE, SV_ERR_BAD_DTYPE):
        raise ValueError(text)
    raise RuntimeError(text)


def as_tensor(x) -> torch.Tensor:
    """Borrow any DLPack-capable array as a torch tensor (zero copy); pass tensors through."""

    if isinstance(x, torch.Tensor):
        return x
    if hasattr(x, "__dlpack__"):
        return torch.from_dlpack(x)
    return torch.as_tensor(x)


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(
            f"{name} must live on a CUDA device: this package runs only on the GPU "
            "(no CPU fallback)"
        )


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream(device: torch.device) -> int:
    """The device's current CUDA stream handle (what torch launches its own kernels on)."""

    if _raw_stream is not None:
        index = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(index)
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Caller-owned scratch from torch's caching allocator (no cudaMalloc in steady state)."""

    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The per-device int32 word kernels OR error bits into."""

    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _status.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _status[index] = word
    return word


def check_device_status(device: torch.device | None = None) -> None:
    """Synchronise, read and clear the device status word; raise if a kernel flagged an error."""

    device = device or torch.device("cuda", torch.cuda.current_device())
    word = status_word(device)
    bits = int(word.item())
    if bits:
        word.zero_()
        parts = []
        if bits & SV_DEVICE_TABLE_FULL:
            parts.append("coordinate hash table full")
        if bits & SV_DEVICE_BAD_INDEX:
            parts.append("neighbour/row index out of range (treated as missing)")
        if bits & SV_DEVICE_WAIT_TIMEOUT:
            parts.append("an in-kernel wait timed out (output invalid)")
        raise RuntimeError("sparsevox device error: " + "; ".join(parts))
