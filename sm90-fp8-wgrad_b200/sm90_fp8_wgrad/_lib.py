"""ctypes binding of the C-ABI library ``libsm100_fp8_wgrad.so``.

The library (built from ``csrc/`` for sm_100a by ``build_ext.py``) is the only
compute path of this package: there is no Python, PyTorch or CPU fallback. A
missing or unloadable library raises ``RuntimeError`` at first use.

The structures below mirror ``include/sm100_fp8_wgrad.h`` field by field.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_NAME = "libsm100_fp8_wgrad.so"
LIB_PATH = Path(__file__).resolve().parent / "_lib" / LIB_NAME

OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED_ARCH = 2
ERR_LAUNCH = 3
ERR_TENSOR_MAP = 4
ERR_DEVICE_TIMEOUT = 5
ERR_UNSUPPORTED = 6

OUT_BF16 = 0
OUT_F32 = 1

TILE_AUTO = 0
TILE_128x256 = 1
TILE_128x128 = 2
TILE_128x256_W8 = 3
TILE_128x256_W16 = 4
TILE_128x128_2CTA = 5
TILE_128x192_W12 = 6
TILE_128x192_UE8M0 = 7
TILE_256x256_PAIR = 8
TILE_256x256_PAIR_W16 = 9
TILE_256x256_SP = 10
TILE_256x256_SP_W16 = 11
SCALE_FP32 = 0
SCALE_UE8M0 = 1

# Every symbol include/sm100_fp8_wgrad.h declares.
EXPORTED_SYMBOLS = (
    "sm100_fp8_grouped_wgrad",
    "sm100_fp8_grouped_wgrad_noalloc",
    "sm100_wgrad_workspace_bytes",
    "sm100_wgrad_quantize_1x128",
    "sm100_wgrad_quantize_1x128_ex",
    "sm100_wgrad_build_meta",
    "sm100_wgrad_device_error",
    "sm100_wgrad_poll_device_error",
    "sm100_wgrad_build_flags",
    "sm100_wgrad_profile_counters",
    "sm100_wgrad_status_string",
    "sm100_wgrad_version",
)


class Sm100WgradArgs(ctypes.Structure):
    _fields_ = [
        ("lhs_data", ctypes.c_void_p),
        ("lhs_pitch", ctypes.c_int64),
        ("lhs_scales", ctypes.c_void_p),
        ("rhs_data", ctypes.c_void_p),
        ("rhs_pitch", ctypes.c_int64),
        ("rhs_scales", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_dtype", ctypes.c_int32),
        ("accumulate", ctypes.c_int32),
        ("num_experts", ctypes.c_int64),
        ("m", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k_rows", ctypes.c_int64),
        ("total_blocks", ctypes.c_int64),
        ("block_offsets", ctypes.c_void_p),
        ("k_row_offsets", ctypes.c_void_p),
        ("expert_order", ctypes.c_void_p),
        ("tile_config", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
    ]


class Sm100WgradQuantArgs(ctypes.Structure):
    """Mirror of Sm100WgradQuantArgs (include/sm100_fp8_wgrad.h)."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("x_dtype", ctypes.c_int32),
        ("cols", ctypes.c_int64),
        ("gather_idx", ctypes.c_void_p),
        ("block_row_start", ctypes.c_void_p),
        ("block_row_count", ctypes.c_void_p),
        ("total_blocks", ctypes.c_int64),
        ("q_data", ctypes.c_void_p),
        ("q_pitch", ctypes.c_int64),
        ("q_row_start", ctypes.c_void_p),
        ("q_zero_fill", ctypes.c_int32),
        ("kq_data", ctypes.c_void_p),
        ("kq_pitch", ctypes.c_int64),
        ("kq_row_start", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("block_rows", ctypes.c_int32),
        ("x_rows", ctypes.c_int64),
        ("scale_format", ctypes.c_int32),
    ]


class Sm100WgradMetaOut(ctypes.Structure):
    _fields_ = [
        ("blocks_per_expert", ctypes.c_void_p),
        ("block_offsets", ctypes.c_void_p),
        ("padded_cu_seqlens_k", ctypes.c_void_p),
        ("wgmma_cu_seqlens_k", ctypes.c_void_p),
        ("tail_valid_rows", ctypes.c_void_p),
        ("tail_wgmma_atoms", ctypes.c_void_p),
        ("tail_copy_k", ctypes.c_void_p),
        ("has_tail", ctypes.c_void_p),
        ("expert_order", ctypes.c_void_p),
        ("block_row_start", ctypes.c_void_p),
        ("block_row_count", ctypes.c_void_p),
        ("wgmma_block_row_start", ctypes.c_void_p),
        ("block_capacity", ctypes.c_int64),
        ("totals", ctypes.c_void_p),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    override = os.environ.get("SM100_WGRAD_LIB")
    return Path(override) if override else LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raise RuntimeError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.is_file():
            raise RuntimeError(
                f"{LIB_NAME} not found at {path}; build it with "
                "`python sm90-fp8-wgrad_b200/build_ext.py` (nvcc, sm_100a)"
            )
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as exc:
            raise RuntimeError(f"cannot load {path}: {exc}") from exc
        lib.sm100_fp8_grouped_wgrad.argtypes = [ctypes.POINTER(Sm100WgradArgs), ctypes.c_void_p]
        lib.sm100_fp8_grouped_wgrad.restype = ctypes.c_int
        lib.sm100_fp8_grouped_wgrad_noalloc.argtypes = [ctypes.POINTER(Sm100WgradArgs), ctypes.c_void_p]
        lib.sm100_fp8_grouped_wgrad_noalloc.restype = ctypes.c_int
        lib.sm100_wgrad_workspace_bytes.argtypes = [ctypes.POINTER(Sm100WgradArgs), ctypes.POINTER(ctypes.c_int64)]
        lib.sm100_wgrad_workspace_bytes.restype = ctypes.c_int
        lib.sm100_wgrad_quantize_1x128.argtypes = [
            ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ]
        lib.sm100_wgrad_quantize_1x128.restype = ctypes.c_int
        lib.sm100_wgrad_quantize_1x128_ex.argtypes = [ctypes.POINTER(Sm100WgradQuantArgs), ctypes.c_void_p]
        lib.sm100_wgrad_quantize_1x128_ex.restype = ctypes.c_int
        lib.sm100_wgrad_build_meta.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(Sm100WgradMetaOut), ctypes.c_void_p,
        ]
        lib.sm100_wgrad_build_meta.restype = ctypes.c_int
        lib.sm100_wgrad_profile_counters.argtypes = [ctypes.POINTER(ctypes.c_uint64), ctypes.c_int32]
        lib.sm100_wgrad_profile_counters.restype = ctypes.c_int
        lib.sm100_wgrad_device_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
        lib.sm100_wgrad_device_error.restype = ctypes.c_int
        lib.sm100_wgrad_poll_device_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
        lib.sm100_wgrad_poll_device_error.restype = ctypes.c_int
        lib.sm100_wgrad_build_flags.argtypes = []
        lib.sm100_wgrad_build_flags.restype = ctypes.c_int
        lib.sm100_wgrad_status_string.argtypes = [ctypes.c_int]
        lib.sm100_wgrad_status_string.restype = ctypes.c_char_p
        lib.sm100_wgrad_version.argtypes = []
        lib.sm100_wgrad_version.restype = ctypes.c_char_p
        _lib = lib
        return lib


def status_string(status: int) -> str:
    return load().sm100_wgrad_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    """Map a non-zero C status to RuntimeError (the reference's error type)."""
    if int(status) != OK:
        raise RuntimeError(f"{what} failed: status {int(status)} ({status_string(status)})")


PROFILE_SLOTS = ("producer_wait_stage", "producer_wait_scales", "mma_wait", "mma_issue", "epi_wait",
                 "epi_promote", "epi_store", "epi_store_wait", "k_blocks", "tiles", "ctas", "sf_convert",
                 "sf_publish", "load_latency", "sf_sync", "sf_load", "mma_tile_wait", "cta_cycles")


def profile_counters() -> dict[str, int] | None:
    """Per-role cycle counters of the grouped GEMM since the last call (read and
    cleared), or None when the loaded library was built without WGRAD_PROFILE
    (build one with ``build_ext.py --profile`` and point SM100_WGRAD_LIB at it)."""
    buf = (ctypes.c_uint64 * 24)()
    status = load().sm100_wgrad_profile_counters(buf, 24)
    if int(status) == ERR_UNSUPPORTED:
        return None
    check(status, "sm100_wgrad_profile_counters")
    return {name: int(buf[i]) for i, name in enumerate(PROFILE_SLOTS)}


def device_error() -> int:
    """Read and clear the device error word of the current device (synchronous)."""
    code = ctypes.c_int32(0)
    check(load().sm100_wgrad_device_error(ctypes.byref(code)), "sm100_wgrad_device_error")
    return int(code.value)


DEVICE_ERRORS = {
    1: "a bounded wait of the GEMM's producer gave up (device-side timeout)",
    2: "a bounded wait of the GEMM's MMA issuer gave up (device-side timeout)",
    3: "a bounded wait of the GEMM's promotion/epilogue warps gave up (device-side timeout)",
    4: "a tile index outside the launch",
    5: "a quantiser gather index outside [0, x_rows)",
    6: "an operand labelled UE8M0 carried a scale that is not a positive power of two",
}

BUILD_DEBUG_MODES = 1
BUILD_PROFILE = 2


def build_flags() -> int:
    """Compile-time features of the loaded library (BUILD_* bit mask)."""
    return int(load().sm100_wgrad_build_flags())


def poll_device_error() -> int:
    """Device error recorded by a finished launch since the last poll or read
    (0 if none), read from a pinned host-mapped word without synchronising."""
    code = ctypes.c_int32(0)
    status = load().sm100_wgrad_poll_device_error(ctypes.byref(code))
    if int(status) == ERR_UNSUPPORTED:
        return 0
    check(status, "sm100_wgrad_poll_device_error")
    return int(code.value)


def raise_device_error(code: int, when: str) -> None:
    if code:
        what = DEVICE_ERRORS.get(int(code), "unknown device error")
        raise RuntimeError(f"sm100 Wgrad device error {int(code)} {when}: {what}; the output of that launch is invalid")


def raise_pending_device_error() -> None:
    """Raise RuntimeError if an earlier launch on the current device recorded a
    device-side error (non-blocking; see poll_device_error)."""
    raise_device_error(poll_device_error(), "in an earlier launch")


def version() -> str:
    return load().sm100_wgrad_version().decode()
