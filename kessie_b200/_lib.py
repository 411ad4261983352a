"""ctypes binding of libkessie_cuda.so (the C ABI declared in include/kessie_capi.h).

The library is the only compute path: there is no CPU or Triton fallback.  If
the shared object is missing, ``load()`` raises ``KessieLibraryError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_double, c_float, c_int, c_int64, c_size_t, c_void_p, c_char_p, POINTER, c_uint32, c_uint64

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_PATHS = [
    os.path.join(HERE, "build", "libkessie_cuda.so"),
    os.path.join(HERE, "build", "libkessie_hip.so"),
]

DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2
DEV_BAD_PAGE_ID, DEV_WAIT_TIMEOUT, DEV_BAD_ARG = 0x1, 0x2, 0x4


class KessieFogBias(ctypes.Structure):
    """C layout of kessie_fog_bias (include/kessie_capi.h)."""
    _fields_ = [("fog_alpha", ctypes.c_float), ("fog_start", ctypes.c_double), ("recall_boost", ctypes.c_float),
                ("recall_bits", ctypes.c_void_p), ("recall_nbits", ctypes.c_int), ("dtype", ctypes.c_int)]


class KessieLibraryError(RuntimeError):
    """The CUDA library is missing or could not be loaded."""


class KessieError(RuntimeError):
    """A library entry point returned a non-zero status."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[status {status}] {msg}")
        self.status = status


P = c_void_p
I32P = c_void_p
# name -> (restype, argtypes); order and types follow include/kessie_capi.h
SIGNATURES = {
    "kessie_get_last_error": (c_int, [c_char_p, c_int]),
    "kessie_version": (c_char_p, []),
    "kessie_read_device_status": (c_int, [P]),
    "kessie_launch_registry_claim": (c_int, [P, P, c_int, P, c_int, c_uint64, c_int, P, P]),
    # legacy (kessie_kernels_v2.hip:714-844)
    "launch_kessie_windowed_attn": (None, [P, P, P, P, c_float, c_int, c_int, c_int, c_int, c_int, c_int, P]),
    "launch_kessie_fused_fog_attn": (None, [P, P, P, P, P, c_float, c_int, c_int, c_int, c_int, c_int, c_int, P]),
    "launch_kessie_page_evict": (None, [P, P, P, c_int, c_int, P]),
    "launch_kessie_page_insert": (None, [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, P]),
    "launch_kessie_rope_remap": (None, [P, P, P, c_float, c_int, c_int, c_int, P]),
    # v2
    "kessie_rope_remap_v2": (c_int, [P, c_int, c_int, c_int, c_int, c_int64, c_int64, I32P, I32P, c_float, P]),
    "kessie_page_evict_workspace_size": (c_size_t, [c_int]),
    "kessie_page_evict_v2": (c_int, [P, I32P, P, c_int, c_int, I32P, I32P, P, c_size_t, P]),
    "kessie_page_list_valid_v2": (c_int, [P, c_int, I32P, I32P, P, c_size_t, P]),
    "kessie_page_insert_v2": (c_int, [P, c_int, c_int64, c_int64, c_int64, c_int64, c_int, c_int, P, P, c_int64,
                                      c_int64, c_int, c_int, c_int, I32P, P, I32P, c_int, I32P, I32P, c_float, P]),
    "kessie_page_gather_v2": (c_int, [P, c_int, c_int64, c_int64, c_int64, c_int64, c_int, c_int, I32P, c_int,
                                      c_int, c_int, P, P, P]),
    "kessie_build_fog_weights_v2": (c_int, [P, c_int, c_int, c_float, P]),
    "kessie_paged_fog_decode_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "kessie_paged_fog_decode_v2": (c_int, [P, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int, c_int,
                                           I32P, c_int64, I32P, I32P, I32P, I32P, c_float, P, c_int, c_float,
                                           c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, c_size_t, P]),
    "kessie_fog_attention_v2": (c_int, [P, P, P, P, c_int, P, c_float, c_int, c_int, c_int, c_int, c_int, c_int,
                                        c_int, P]),
    "kessie_paged_fog_prefill_v2": (c_int, [P, c_int64, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int,
                                            c_int, I32P, c_int64, I32P, I32P, I32P, c_float, P, c_int64, c_int,
                                            c_int, c_float, c_int, c_int, c_int, c_int, c_int, c_int, P, c_int64,
                                            c_int64, c_int64, P]),
    "kessie_paged_fog_decode_ex_v2": (c_int, [P, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int, c_int,
                                              I32P, c_int64, I32P, I32P, I32P, I32P, c_float, P, c_int, c_float,
                                              c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, c_size_t, c_int, P]),
    "kessie_paged_fog_decode_noalloc_v2": (c_int, [P, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int,
                                                   c_int, I32P, c_int64, I32P, I32P, I32P, I32P, c_float, P, c_int,
                                                   c_float, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P]),
    "kessie_paged_fog_prefill_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "kessie_paged_fog_prefill_ex_v2": (c_int, [P, c_int64, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int,
                                               c_int, I32P, c_int64, I32P, I32P, I32P, c_float, P, c_int64, c_int,
                                               c_int, c_float, c_int, c_int, c_int, c_int, c_int, c_int, P, c_int64,
                                               c_int64, c_int64, c_int, P, c_size_t, P]),
    "kessie_lse_combine_v2": (c_int, [P, c_int, c_int64, c_int, c_int, P, c_int, P, P]),
    "kessie_build_fog_bias_v2": (c_int, [P, c_int, c_int, P, P]),
    "kessie_index_query_workspace_size": (c_size_t, [c_int, c_int]),
    "kessie_index_query_v2": (c_int, [P, P, c_int, c_int, c_int, P, c_int, P, P, P, c_size_t, P]),
    "kessie_tiered_update_v2": (c_int, [P, P, c_int64, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int, c_int,
                                        c_int, c_int, c_int, P, c_float, c_double, P]),
    "kessie_strided_pack_v2": (c_int, [P, P, c_int, c_int, c_int64, c_int, P, c_int, P]),
    "kessie_paged_fog_decode_biased_v2": (c_int, [P, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int, c_int,
                                                  I32P, c_int64, I32P, I32P, I32P, I32P, c_float, P, c_int, c_float,
                                                  c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, c_size_t, P]),
    "kessie_paged_fog_prefill_biased_v2": (c_int, [P, c_int64, c_int64, c_int64, P, P, c_int64, c_int64, c_int64,
                                                   c_int, c_int, I32P, c_int64, I32P, I32P, c_int, c_int, c_float,
                                                   c_int, c_int, c_int, c_int, c_int, c_int, P, P, c_int64, c_int64,
                                                   c_int64, c_int, P, c_size_t, P]),
    "kessie_cp_exchange_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "kessie_cp_exchange_alloc": (c_int, [c_size_t, P, P]),
    "kessie_cp_exchange_open": (c_int, [P, P]),
    "kessie_cp_exchange_close": (c_int, [P]),
    "kessie_cp_exchange_free": (c_int, [P]),
    "kessie_cp_combine_v2": (c_int, [P, c_int, c_int, c_uint32, c_int64, c_int, c_int, c_int, c_int, c_int, P, P, P]),
    "kessie_paged_fog_decode_cp_v2": (c_int, [P, c_int64, c_int64, P, P, c_int64, c_int64, c_int64, c_int, c_int,
                                              I32P, c_int64, I32P, I32P, I32P, I32P, c_float, P, c_int, c_float,
                                              c_int, c_int, c_int, c_int, c_int, c_int, P, c_int, c_int, c_uint32,
                                              c_int64, P, P, P, c_size_t, c_int, P]),
}

_lock = threading.Lock()
_lib = None
_path = None


def library_path() -> str:
    env = os.environ.get("KESSIE_LIB")
    cands = ([env] if env else []) + DEFAULT_PATHS
    for p in cands:
        if p and os.path.exists(p):
            return p
    raise KessieLibraryError(
        "libkessie_cuda.so not found; build it with `python -m kessie_b200.build` "
        f"(searched {cands})")


def load():
    """Load (once) and return the ctypes library with signatures set."""
    global _lib, _path
    with _lock:
        if _lib is None:
            path = library_path()
            try:
                lib = ctypes.CDLL(path)
            except OSError as e:
                raise KessieLibraryError(f"cannot load {path}: {e}") from e
            for name, (res, args) in SIGNATURES.items():
                try:
                    fn = getattr(lib, name)
                except AttributeError:
                    continue        # reported by missing_symbols(); calling it raises AttributeError
                fn.restype = res
                fn.argtypes = args
            _lib, _path = lib, path
        return _lib


_binding = None


def load_binding():
    """The torch extension module `kessie_hip` (kessie_b200/build/kessie_hip.so):
    the reference's pybind11 boundary (kessie_hip_binding.cpp:216-239) over
    this library.  Loads libkessie_cuda.so globally first, since the module
    resolves the launchers from it."""
    global _binding
    with _lock:
        if _binding is None:
            import importlib.machinery
            import importlib.util
            import sys
            import torch  # noqa: F401  (the module links against libtorch)
            path = os.path.join(HERE, "build", "kessie_hip.so")
            if not os.path.exists(path):
                raise KessieLibraryError(f"{path} not found; build it with `python -m kessie_b200.build`")
            ctypes.CDLL(library_path(), mode=ctypes.RTLD_GLOBAL)
            loader = importlib.machinery.ExtensionFileLoader("kessie_hip", path)
            spec = importlib.util.spec_from_loader("kessie_hip", loader)
            mod = importlib.util.module_from_spec(spec)
            loader.exec_module(mod)
            sys.modules.setdefault("kessie_hip", mod)
            _binding = mod
        return _binding


def missing_symbols():
    lib = load()
    return [n for n in SIGNATURES if not hasattr(lib, n)]


def loaded_path():
    return _path


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    st = load().kessie_get_last_error(buf, 512)
    return st, buf.value.decode(errors="replace")


def check(status: int, what: str = ""):
    if status != 0:
        st, msg = last_error()
        raise KessieError(status, f"{what}: {msg}" if what else msg)


def check_legacy(what: str):
    """Legacy launchers return void; a failure is left in the last-error slot."""
    st, msg = last_error()
    if st != 0:
        raise KessieError(st, f"{what}: {msg}")
