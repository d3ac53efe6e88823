"""The C ABI library loads and exports every function include/*.h declares
(no GPU: nothing here launches a kernel)."""
import glob
import os
import re
import subprocess

import pytest

import charlotte_b200 as cb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        names.update(re.findall(r"CB_API\s+[\w\s\*]+?\b(cb_\w+)\s*\(", text))
    return sorted(names)


def test_headers_declare_functions():
    assert "cb_matmul_run" in declared_functions()


def test_library_exports_every_declared_function():
    out = subprocess.run(["nm", "-D", "--defined-only", cb.library_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s(cb_\w+)$", out, re.M))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing


def test_library_loads_and_names_itself():
    L = cb.lib()
    for name in declared_functions():
        assert hasattr(L, name)
    assert L.cb_version().decode().count(".") == 2


def test_invalid_arguments_are_a_status_not_a_fault():
    """Argument checks run before any device work: no GPU needed."""
    import ctypes
    m = cb.Matmul()
    m.format = 6            # Q5_0: no kernel here
    m.columns = 64
    m.members = 1
    outs = (ctypes.c_void_p * 3)(1, 0, 0)
    st = (ctypes.c_uint32 * 3)(0, 0, 0)
    rc = cb.lib().cb_matmul_run(ctypes.byref(m), 16, 64, 1, ctypes.byref(outs), ctypes.byref(st), 0, None)
    assert rc == cb.ERROR_INVALID and "format 6" in cb.last_error()
    m.format = cb.Q4_0
    m.columns = 33
    rc = cb.lib().cb_matmul_run(ctypes.byref(m), 16, 64, 1, ctypes.byref(outs), ctypes.byref(st), 0, None)
    assert rc == cb.ERROR_INVALID and "32-weight" in cb.last_error()


@pytest.mark.parametrize("fmt", [2, 3, 8, 14, 30])   # Q4_0, Q4_1, Q8_0, Q6_K, BF16
def test_piece_from_stored_is_the_device_layout(fmt):
    """cb_piece_from_stored (host code, no GPU) writes the device layout the
    kernels read: the same bytes as the oracle's layout of the same blocks."""
    import ctypes
    import numpy as np
    import oracle as O
    from charlotte_b200 import synth
    rng = np.random.default_rng(fmt)
    stored = synth.random_bytes_blocks(rng, fmt, 64 if fmt != 30 else 640)
    blocks = stored.size // O.BLOCK_BYTES[fmt]
    L = cb.lib()
    L.cb_piece_bytes.restype = ctypes.c_size_t
    L.cb_piece_bytes.argtypes = [ctypes.c_uint32, ctypes.c_uint64]
    out = np.zeros(L.cb_piece_bytes(fmt, blocks), np.uint8)
    L.cb_piece_from_stored.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
    assert L.cb_piece_from_stored(fmt, stored.ctypes.data, blocks, out.ctypes.data) == 0
    assert np.array_equal(out, O.to_piece(fmt, stored))


@pytest.mark.parametrize("fn", ["cb_select_run", "cb_select_run_static"])
def test_select_refuses_ids_past_32_bits(fn):
    """Both selection entry points share one argument check: ids of a
    vocabulary shard (id_offset + count) past 2^32 - 1 would wrap into the
    padding id, so they are refused before anything runs (no GPU)."""
    import ctypes
    s = cb.Select()
    s.logits, s.candidates, s.sampled = 16, 16, 16
    if fn == "cb_select_run":
        s.partials, s.ticket = 16, 16
    s.count = 1024
    s.id_offset = 0xFFFFFFFF - 1000
    rc = getattr(cb.lib(), fn)(ctypes.byref(s), 0, None)
    assert rc == cb.ERROR_INVALID and "2^32" in cb.last_error()
    # candidates_only with no record is accepted by the checks of both
    s.id_offset = 0
    s.count = 0
    s.sampled = 0
    s.candidates_only = 1
    rc = getattr(cb.lib(), fn)(ctypes.byref(s), 0, None)
    assert rc == cb.ERROR_INVALID and "entries" in cb.last_error()


def test_integration_library_exports_the_boundary():
    """integration/libcharlotte_program.so (the CUDA Upload and Program built
    with the reference's loader, plan and launchers) loads beside the
    library and exports its harness (no GPU: nothing runs)."""
    import ctypes
    lib = os.path.join(ROOT, "integration", "libcharlotte_program.so")
    if not os.path.exists(lib):
        pytest.skip("the reference sources were absent when it would have been built")
    cb.lib()
    L = ctypes.CDLL(lib)
    for name in ("cbh_open", "cbh_run", "cbh_poll", "cbh_logits", "cbh_profile", "cbh_close"):
        assert hasattr(L, name)
