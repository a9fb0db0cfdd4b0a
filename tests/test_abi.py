"""The C-ABI library loads and exports every declared symbol (no GPU, no compute)."""
import ctypes
import os
import re

import insitu_b200 as ib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("insitu_b200.h", "cuda_wrapper.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M):
            if m.group(1) not in ("defined",):
                names.add(m.group(1))
    return names


def test_headers_declare_the_binding_list():
    assert declared_functions() == set(ib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(ib.library_path())
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_no_device_calls_fail_cleanly():
    lib = ib.load_library(require_device=False)
    import torch

    if torch.cuda.is_available():
        return
    assert lib.cuda_is_available() is False
    assert lib.ivf_create_batch_context(16, 32, 4, 4, 8) is None
    assert lib.ivf_global_last_error().decode() != ""
    # a null / foreign context is rejected, not dereferenced blindly
    assert lib.ivf_route(None, None, 1, 1) == -1
    assert lib.ivf_check_index_initialized_wrapper(None) == 0
    assert lib.ivf_pq_delta_mode(None) == -1
