"""ctypes binding of libamq4.so (the C ABI declared in include/am_q4.h).

The shared library is built in-tree (see ``build.py``) and loaded from this package
directory.  There is no fallback: if the library is missing or cannot be loaded, every
kernel entry point raises :class:`Q4KernelUnavailable`.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_NAME = "libamq4.so"
LIB_PATH = PKG_DIR / LIB_NAME

ABI_VERSION = 4

# Status codes / enums (mirrors include/am_q4.h)
AM_OK = 0
AM_ERR_INVALID = -1
AM_ERR_UNSUPPORTED = -2
AM_ERR_WORKSPACE = -3
AM_ERR_CUDA = -4

DTYPE_F16, DTYPE_BF16, DTYPE_F32, DTYPE_U8 = 0, 1, 2, 3
LAYOUT_CONTIGUOUS, LAYOUT_PAGED = 0, 1
MASK_NONE, MASK_BOOL, MASK_ADDITIVE = 0, 1, 2
STATUS_BAD_BLOCK, STATUS_BAD_POSITION, STATUS_TIMEOUT, STATUS_POOL_EXHAUSTED = 1, 2, 4, 8

EXPORTED_SYMBOLS = (
    "am_abi_version",
    "am_last_error",
    "am_q4_quantize",
    "am_q4_dequantize",
    "am_q4_append",
    "am_q4_decode_workspace_bytes",
    "am_q4_prefill_workspace_bytes",
    "am_q4_attention_workspace_bytes",
    "am_q4_decode",
    "am_q4_prefill",
    "am_q4_prefill_stage",
    "am_q4_prefill_attend",
    "am_q4_attention",
    "am_q4_decode_noalloc",
    "am_q4_blocks_pack",
    "am_q4_blocks_unpack",
    "am_block_reserve",
    "am_block_release",
)
STATIC_DECODE_SCRATCH_BYTES = 16 << 20

c_void_p, c_int32, c_int64, c_float, c_size_t = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                                 ctypes.c_float, ctypes.c_size_t)


class Q4CacheDesc(ctypes.Structure):
    """Mirror of ``am_q4_cache``."""

    _fields_ = [
        ("k_codes", c_void_p),
        ("k_scales", c_void_p),
        ("k_biases", c_void_p),
        ("v_codes", c_void_p),
        ("v_scales", c_void_p),
        ("v_biases", c_void_p),
        ("scale_dtype", c_int32),
        ("layout", c_int32),
        ("n_kv_heads", c_int32),
        ("k_dim", c_int32),
        ("v_dim", c_int32),
        ("block_tokens", c_int32),
        ("capacity", c_int64),
        ("batch", c_int32),
        ("block_table_stride", c_int32),
        ("block_table", c_void_p),
    ]


class AttnArgs(ctypes.Structure):
    """Mirror of ``am_attn_args``."""

    _fields_ = [
        ("q", c_void_p),
        ("q_dtype", c_int32),
        ("batch", c_int32),
        ("n_q_heads", c_int32),
        ("q_len", c_int32),
        ("q_stride_b", c_int64),
        ("q_stride_h", c_int64),
        ("q_stride_l", c_int64),
        ("out", c_void_p),
        ("out_dtype", c_int32),
        ("causal", c_int32),
        ("o_stride_b", c_int64),
        ("o_stride_h", c_int64),
        ("o_stride_l", c_int64),
        ("scale", c_float),
        ("window", c_int32),
        ("kv_len", c_void_p),
        ("kv_start", c_void_p),
        ("max_kv_len", c_int32),
        ("mask_kind", c_int32),
        ("mask", c_void_p),
        ("mask_dtype", c_int32),
        ("reserved0", c_int32),
        ("mask_stride_b", c_int64),
        ("mask_stride_h", c_int64),
        ("mask_stride_l", c_int64),
        ("mask_stride_n", c_int64),
        ("status", c_void_p),
        ("sinks", c_void_p),
    ]


class Q4KernelUnavailable(RuntimeError):
    """The CUDA library could not be loaded; there is no CPU path to fall back to."""


class Q4KernelError(RuntimeError):
    """A library call returned an error status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load libamq4.so once and declare its signatures.  Raises Q4KernelUnavailable."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    if path is None and os.environ.get("AM_Q4_LIB"):
        path = os.environ["AM_Q4_LIB"]  # an alternative build of the same library
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise Q4KernelUnavailable(
            f"{p} is missing: build it with `python -m agent_memory_b200.build` (nvcc, sm_100a)")
    try:
        lib = ctypes.CDLL(str(p))
    except OSError as e:  # pragma: no cover - depends on the host
        raise Q4KernelUnavailable(f"cannot load {p}: {e}") from e
    for sym in EXPORTED_SYMBOLS:
        if not hasattr(lib, sym):
            raise Q4KernelUnavailable(f"{p} does not export {sym}")
    lib.am_abi_version.restype = c_int32
    lib.am_last_error.restype = ctypes.c_char_p
    lib.am_q4_quantize.argtypes = [c_void_p, c_int32, c_int64, c_int32, c_void_p, c_void_p,
                                   c_void_p, c_void_p]
    lib.am_q4_quantize.restype = c_int32
    lib.am_q4_dequantize.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_int32,
                                     c_void_p, c_int32, c_void_p]
    lib.am_q4_dequantize.restype = c_int32
    lib.am_q4_append.argtypes = [ctypes.POINTER(Q4CacheDesc), c_void_p, c_void_p, c_int32, c_int32,
                                 c_int32, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                                 c_void_p, c_void_p, c_void_p]
    lib.am_q4_append.restype = c_int32
    for fn in ("am_q4_decode_workspace_bytes", "am_q4_prefill_workspace_bytes",
               "am_q4_attention_workspace_bytes"):
        f = getattr(lib, fn)
        f.argtypes = [ctypes.POINTER(Q4CacheDesc), ctypes.POINTER(AttnArgs)]
        f.restype = c_size_t
    for fn in ("am_q4_decode", "am_q4_prefill", "am_q4_prefill_attend", "am_q4_attention"):
        f = getattr(lib, fn)
        f.argtypes = [ctypes.POINTER(Q4CacheDesc), ctypes.POINTER(AttnArgs), c_void_p, c_size_t,
                      c_void_p]
        f.restype = c_int32
    lib.am_q4_prefill_stage.argtypes = [ctypes.POINTER(Q4CacheDesc), ctypes.POINTER(AttnArgs),
                                        c_int32, c_int32, c_void_p, c_size_t, c_void_p]
    lib.am_q4_prefill_stage.restype = c_int32
    lib.am_q4_decode_noalloc.argtypes = [ctypes.POINTER(Q4CacheDesc), ctypes.POINTER(AttnArgs),
                                         c_void_p]
    lib.am_q4_decode_noalloc.restype = c_int32
    for fn in ("am_q4_blocks_pack", "am_q4_blocks_unpack"):
        f = getattr(lib, fn)
        f.argtypes = [ctypes.POINTER(Q4CacheDesc), c_void_p, c_void_p, c_void_p, c_int32, c_void_p,
                      c_void_p, c_void_p]
        f.restype = c_int32
    lib.am_block_reserve.argtypes = [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32,
                                     c_void_p, c_void_p, c_int32, c_void_p, c_void_p]
    lib.am_block_reserve.restype = c_int32
    lib.am_block_release.argtypes = [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32,
                                     c_void_p, c_void_p, c_void_p]
    lib.am_block_release.restype = c_int32
    ver = lib.am_abi_version()
    if ver != ABI_VERSION:
        raise Q4KernelUnavailable(f"{p} has ABI version {ver}, expected {ABI_VERSION}")
    _lib = lib
    return lib


def check(fn: str, rc: int) -> None:
    if rc != AM_OK:
        msg = load().am_last_error()
        raise Q4KernelError(fn, rc, msg.decode() if msg else "")
