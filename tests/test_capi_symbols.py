"""CPU: the C-ABI library builds, loads without a GPU, and exports every
entry point include/kessie_capi.h declares, with ctypes signatures set."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kessie_capi.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s+([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_reference_launchers():
    names = declared_functions()
    for legacy in ["launch_kessie_windowed_attn", "launch_kessie_fused_fog_attn", "launch_kessie_page_evict",
                   "launch_kessie_page_insert", "launch_kessie_rope_remap"]:
        assert legacy in names


def test_library_exports_every_declared_symbol():
    from kessie_b200 import _lib
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # every declared symbol has a ctypes signature in the binding
    assert set(declared_functions()) <= set(_lib.SIGNATURES), set(declared_functions()) - set(_lib.SIGNATURES)
    assert b"sm_100a" in lib.kessie_version()


def test_legacy_name_alias_exists():
    from kessie_b200 import _lib
    p = os.path.join(os.path.dirname(_lib.__file__), "build", "libkessie_hip.so")
    assert os.path.exists(p)
    lib = ctypes.CDLL(p)
    assert hasattr(lib, "launch_kessie_fused_fog_attn")


def test_argument_errors_are_reported_without_gpu():
    """Argument validation happens before any CUDA call."""
    from kessie_b200 import _lib
    lib = _lib.load()
    rc = lib.kessie_rope_remap_v2(None, 7, 4, 2, 128, 256, 128, None, None, 1e4, None)
    assert rc == 2
    st, msg = _lib.last_error()
    assert st == 2 and "dtype" in msg
    rc = lib.kessie_paged_fog_decode_v2(None, 0, 0, None, None, 0, 0, 0, 1, 16, None, 0, None, None, None, None,
                                        0.5, None, 0, 0.1, 1, 8, 2, 96, 128, 1, None, None, None, 0, None)
    assert rc == 2  # head_dim 96 unsupported
    assert lib.kessie_page_evict_workspace_size(8192) >= 8192


def test_index_query_and_tiered_cache_argument_errors_without_gpu():
    """The index-query, tiered-update and strided-pack entry points reject bad
    arguments (with a message) before any CUDA call; the fog-start argument of
    the tiered update is a double, as the reference's int(S * fog_start) is."""
    from kessie_b200 import _lib
    lib = _lib.load()
    ERR_ARG = 1                                   # KESSIE_ERR_ARG
    # dim not a multiple of 4
    assert lib.kessie_index_query_v2(16, 16, 100, 6, 1, None, 5, 16, 16, None, 0, None) == ERR_ARG
    assert "dim" in _lib.last_error()[1]
    # top_k above 32
    assert lib.kessie_index_query_v2(16, 16, 100, 8, 1, None, 33, 16, 16, None, 0, None) == ERR_ARG
    # misaligned index
    assert lib.kessie_index_query_v2(16, 20, 100, 8, 1, 16, 0, None, None, None, 0, None) == ERR_ARG
    assert "aligned" in _lib.last_error()[1]
    # nothing requested
    assert lib.kessie_index_query_v2(16, 16, 100, 8, 1, None, 0, None, None, None, 0, None) == ERR_ARG
    # tiered update: hi + T beyond the store
    assert lib.kessie_tiered_update_v2(16, 16, 100, 0, 99, 16, 16, 0, 0, 128, 1, 8, 2, 128, 1, None, 0.5, 0.5,
                                       None) == ERR_ARG
    assert "cap" in _lib.last_error()[1]
    # head_dim * element size not a multiple of 16
    assert lib.kessie_tiered_update_v2(16, 16, 100, 0, 10, 16, 16, 0, 0, 12, 1, 8, 1, 12, 0, None, 0.5, 0.5,
                                       None) == ERR_ARG
    # unaligned store
    assert lib.kessie_tiered_update_v2(24, 16, 100, 0, 10, 16, 16, 0, 0, 128, 1, 8, 1, 128, 1, None, 0.5, 0.5,
                                       None) == ERR_ARG
    assert _lib.SIGNATURES["kessie_tiered_update_v2"][1][17] is ctypes.c_double
    # strided pack: row bytes not a multiple of 16
    assert lib.kessie_strided_pack_v2(16, 16, 2, 8, 10, 24, 16, 0, None) == ERR_ARG
    assert lib.kessie_strided_pack_v2(None, 16, 2, 8, 10, 32, 16, 0, None) == ERR_ARG


LEGACY = ["launch_kessie_windowed_attn", "launch_kessie_fused_fog_attn", "launch_kessie_page_evict",
          "launch_kessie_page_insert", "launch_kessie_rope_remap"]


def header_param_ctypes(name):
    """ctypes types of a legacy launcher's parameters as include/kessie_capi.h
    declares them (pointer -> c_void_p, float -> c_float, int -> c_int)."""
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    m = re.search(r"void\s+" + name + r"\s*\(([^)]*)\)", src)
    assert m, name
    out = []
    for p in m.group(1).split(","):
        p = p.strip()
        out.append(ctypes.c_void_p if "*" in p else ctypes.c_float if p.startswith("float") else ctypes.c_int)
    return out


def test_reference_ctypes_class_binds_this_library():
    """The reference's own, unmodified KeSSieKernels (kessie_hip_ctypes.py:42-114)
    loads this library under the name it searches for and binds all five
    launchers; the argument types it sets are the ones the header declares.
    Needs the reference tree: set KESSIE_REF to its directory."""
    import importlib.util
    import sys
    ref = os.environ.get("KESSIE_REF")
    if not ref or not os.path.exists(os.path.join(ref, "kessie_hip_ctypes.py")):
        pytest.skip("KESSIE_REF (the reference source tree) is not set")
    lib_path = os.path.join(ROOT, "kessie_b200", "build", "libkessie_hip.so")
    old = sys.dont_write_bytecode
    sys.dont_write_bytecode = True            # the reference tree is read-only
    try:
        spec = importlib.util.spec_from_file_location("kessie_ref_hip_ctypes",
                                                      os.path.join(ref, "kessie_hip_ctypes.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        sys.dont_write_bytecode = old
    kernels = mod.KeSSieKernels(lib_path=lib_path)
    for name in LEGACY:
        fn = getattr(kernels.lib, name)
        assert fn.restype is None, name
        assert list(fn.argtypes) == header_param_ctypes(name), name


def test_torch_extension_binding_surface():
    """The torch extension module kessie_hip exposes the reference binding's
    five functions (kessie_hip_binding.cpp:216-239) with its argument names and
    defaults; importing it needs no GPU."""
    from kessie_b200 import _lib
    m = _lib.load_binding()
    want = {
        "windowed_attention": ["Q", "K", "V", "window_size", "causal"],
        "fused_fog_attention": ["Q", "K", "V", "fog_weights", "window_size", "causal"],
        "rope_remap": ["k_data", "orig_positions", "target_positions", "rope_theta"],
        "page_evict": ["page_valid", "page_positions", "evict_before_pos"],
        "page_insert": ["kv_cache", "new_keys", "new_values", "target_page_ids", "page_valid", "page_positions",
                        "insert_conv_position"],
    }
    for name, args in want.items():
        sig = getattr(m, name).__doc__.splitlines()[0]
        got = re.findall(r"(\w+):", sig[sig.index("(") + 1:sig.rindex(")")])
        assert got == args, (name, sig)
    assert "window_size: typing.SupportsInt = 0" in m.windowed_attention.__doc__ or \
        "window_size: int = 0" in m.windowed_attention.__doc__
    assert "rope_theta" in m.rope_remap.__doc__ and "10000.0" in m.rope_remap.__doc__
