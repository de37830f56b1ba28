"""Loader for the native libraries built from ``cuda-kernel_b200/csrc``.

``lib()`` returns the product library (``libswiglu_b200.so``, C ABI in
``include/swiglu_b200.h``) with every entry point typed; ``cublas_lib()`` the
cuBLAS GemmEx baseline. There is no fallback: if a library is missing the
import fails loudly with the command that builds it.
"""
from __future__ import annotations

import ctypes
import subprocess
import threading
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]          # cuda-kernel_b200/
REPO_ROOT = PKG_ROOT.parent
LIB_DIR = PKG_ROOT / "lib"
LIB_PATH = LIB_DIR / "libswiglu_b200.so"
CUBLAS_LIB_PATH = LIB_DIR / "libswiglu_b200_cublas.so"
TIMELINE_LIB_PATH = LIB_DIR / "libswiglu_b200_timeline.so"   # measurement build (make timeline)
HEADERS = [REPO_ROOT / "include" / "swiglu_b200.h", REPO_ROOT / "include" / "swiglu_b200_cublas.h"]

# status codes (include/swiglu_b200.h)
SWB_OK = 0
SWB_E_INPUT = 1
SWB_E_GATE_BUFFERS = 2
SWB_E_HALF_OUTPUT = 3
SWB_E_FLOAT_OUTPUT = 4
SWB_E_RESIDUAL = 5
SWB_E_CONFIG = 6
SWB_E_SHAPE = 7
SWB_E_CONFIG_RANGE = 8
SWB_E_CONFIG_INVALID = 9
SWB_E_OVERLAP_INPUT = 10
SWB_E_OVERLAP_OUTPUT = 11
SWB_E_CUDA = 12
SWB_E_DEVICE = 13
SWB_E_UNSUPPORTED = 14
SWB_E_WORKSPACE = 15
SWB_NOALLOC_MAX_INTER = 65536
SWB_TP_MAX_RANKS = 8
SWB_LAYER_WORKSPACE_BYTES = 8192
SWB_TP_HANDLE_BYTES = 64
SWB_DEVERR_PEER_TIMEOUT = 2
SWB_PREFETCH_WEIGHTS = 1
SWB_RESIDUAL = 1
SWB_HALF_OUT = 2
SWB_FAMILY_LDG = 0
SWB_FAMILY_BULK = 1
SWB_FAMILY_RBULK = 2
SWB_FAMILY_SBULK = 3
SWBL_E_CUBLAS = 100


class SwbConfig(ctypes.Structure):
    """swb_config_t: host metadata of one registry geometry."""
    _fields_ = [(name, ctypes.c_int) for name in
                ("id", "family", "warps", "rows", "pack", "unroll", "chunk", "stages")]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class NativeLibraryMissing(RuntimeError):
    pass


def build(jobs: int = 2) -> None:
    """Compile both libraries for sm_100a in-tree (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", str(PKG_ROOT)], check=True)


_lock = threading.Lock()
_lib = None
_cublas = None

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64


def _declare(L: ctypes.CDLL) -> ctypes.CDLL:
    sig = {
        "swb_status_string": ([_i], ctypes.c_char_p),
        "swb_last_error": ([], ctypes.c_char_p),
        "swb_version": ([], _i),
        "swb_cuda_versions": ([ctypes.POINTER(_i), ctypes.POINTER(_i)], _i),
        "swb_config_count": ([], _i),
        "swb_config_ids": ([ctypes.POINTER(_i), _i], _i),
        "swb_valid_config": ([_i64], _i),
        "swb_config_info": ([_i64, ctypes.POINTER(SwbConfig)], _i),
        "swb_gate": ([_i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp], _i),
        "swb_project": ([_i, _vp, _vp, _vp, _vp, _vp, _i, _i, ctypes.c_uint, _vp], _i),
        "swb_ffn": ([_i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp], _i),
        "swb_ffn_ex": ([_i, _i] + [_vp] * 9 + [_i, _i, ctypes.c_uint, _vp], _i),
        "swb_ffn_tp": ([_i, _i] + [_vp] * 8 + [_i, _i, _vp], _i),
        "swb_ffn_noalloc": ([_i, _i] + [_vp] * 8 + [_i, _i, _vp], _i),
        "swb_layer_config_count": ([], _i),
        "swb_layer_config_ids": ([ctypes.POINTER(_i), _i], _i),
        "swb_ffn_fused": ([_i] + [_vp] * 9 + [_i, _i, _vp, _vp], _i),
        "swb_ffn_fused_ex": ([_i] + [_vp] * 9 + [_i, _i, _vp, ctypes.c_uint, _vp], _i),
        "swb_swiglu_out": ([_vp] * 6 + [_i64] * 4 + [_vp], _i),
        "swb_tp_create": ([_i, _i, _i, ctypes.POINTER(_vp)], _i),
        "swb_tp_ipc_handle": ([_vp, _vp], _i),
        "swb_tp_connect": ([_vp, _vp], _i),
        "swb_tp_destroy": ([_vp], _i),
        "swb_tp_epoch": ([_vp, ctypes.POINTER(ctypes.c_uint32)], _i),
        "swb_ffn_tp_fused": ([_vp, _i, _i] + [_vp] * 9 + [_i, _i, _vp], _i),
        "swb_ffn_tp_fused_ex": ([_vp, _i, _i] + [_vp] * 9 + [_i, _i, ctypes.c_uint, _vp], _i),
        "swb_ffn_host_ex": ([_i, _i] + [_vp] * 11 + [_i, _i, ctypes.c_uint, _vp], _i),
        "swb_ffn_tp_host_ex": ([_vp, _i, _i] + [_vp] * 11 + [_i, _i, ctypes.c_uint, _vp], _i),
        "swb_swiglu_tp_out": ([_vp] * 7 + [_i64] * 4 + [ctypes.c_uint, _vp], _i),
        "swb_gate_epilogue": ([_vp, _vp, _vp, _vp, _vp, _i, _vp], _i),
        "swb_residual_epilogue": ([_vp, _vp, _vp, _i, _vp], _i),
        "swb_device_error": ([_i, ctypes.POINTER(_i)], _i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    return L


def _declare_cublas(L: ctypes.CDLL) -> ctypes.CDLL:
    sig = {
        "swbl_create": ([ctypes.POINTER(_vp)], _i),
        "swbl_destroy": ([_vp], _i),
        "swbl_last_error": ([], ctypes.c_char_p),
        "swbl_version": ([_vp, ctypes.POINTER(_i)], _i),
        "swbl_gemv": ([_vp, _i, _vp, _vp, _vp, _i, _i, _vp], _i),
        "swbl_ffn": ([_vp, _i] + [_vp] * 11 + [_i, _i, _vp], _i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    return L


def lib() -> ctypes.CDLL:
    """The product library; raises NativeLibraryMissing if it was never built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise NativeLibraryMissing(
                        f"{LIB_PATH} is missing: build it with `make -C {PKG_ROOT}` "
                        "(or __graft_entry__.build()); there is no CPU fallback")
                _lib = _declare(ctypes.CDLL(str(LIB_PATH)))
    return _lib


def cublas_lib() -> ctypes.CDLL:
    global _cublas
    if _cublas is None:
        with _lock:
            if _cublas is None:
                if not CUBLAS_LIB_PATH.exists():
                    raise NativeLibraryMissing(f"{CUBLAS_LIB_PATH} is missing: build it with `make -C {PKG_ROOT}`")
                _cublas = _declare_cublas(ctypes.CDLL(str(CUBLAS_LIB_PATH)))
    return _cublas


def timeline_lib(path=None) -> ctypes.CDLL:
    """The timeline measurement build (``make timeline``): the product's C ABI plus
    swb_timeline_reset/read/capacity. Used only by swiglu_b200.timeline."""
    path = Path(path) if path else TIMELINE_LIB_PATH
    if not path.exists():
        raise NativeLibraryMissing(f"{path} is missing: build it with `make -C {PKG_ROOT} timeline`")
    L = _declare(ctypes.CDLL(str(path)))
    L.swb_timeline_reset.argtypes, L.swb_timeline_reset.restype = [], _i
    L.swb_timeline_read.argtypes, L.swb_timeline_read.restype = [_vp, ctypes.POINTER(ctypes.c_uint)], _i
    L.swb_timeline_capacity.argtypes, L.swb_timeline_capacity.restype = [], _i
    return L


def status_message(status: int) -> str:
    return lib().swb_status_string(int(status)).decode()


def last_error() -> str:
    return lib().swb_last_error().decode()


def check(status: int) -> None:
    """Raise RuntimeError with the library's message for a non-zero status."""
    if status:
        msg = last_error() or status_message(status)
        raise RuntimeError(msg)


def declared_signatures() -> dict[str, int]:
    """Number of parameters of every function the public headers declare."""
    import re
    out = {}
    for h in HEADERS:
        text = h.read_text()
        for m in re.finditer(r"^SWB_API\s+(?:const\s+)?\w+\*?\s+(\w+)\(([^;]*?)\);", text, flags=re.M | re.S):
            params = " ".join(m.group(2).split())
            out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def declared_symbols() -> list[str]:
    """Every function the public headers declare (for export checks)."""
    import re
    names = []
    for h in HEADERS:
        names += re.findall(r"^SWB_API\s+(?:const\s+)?\w+\*?\s+(\w+)\(", h.read_text(), flags=re.M)
    return names
