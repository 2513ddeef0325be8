"""The C-ABI library builds for sm_100a, loads without a GPU, and exports every symbol include/vllm_turing_b200.h
declares, with a ctypes signature for each. CPU only (no compute calls)."""
import ctypes
import os
import re
import subprocess

from vllm_turing_b200 import _build

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "vllm_turing_b200.h")


def header_symbols():
    text = open(HDR).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:unsigned|int|size_t|void|long long)\s*\**\s*(\w+)\s*\(", text, re.M)))


def test_header_parses():
    syms = header_symbols()
    for s in ("w8a8_gemv", "vt_all_reduce", "vt_tp_row_linear", "ce_alloc", "vt_comm_create", "silu_mul_quant"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    so = _build.load()._name
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in header_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_every_declared_symbol_has_a_ctypes_signature():
    missing = [s for s in header_symbols() if s not in _build.SIGNATURES]
    assert not missing, missing
    L = _build.load()
    for s in header_symbols():
        fn = getattr(L, s)
        assert fn.argtypes is not None, s


def test_library_is_current_and_built_for_sm100a():
    assert _build.is_current()
    assert ("-gencode", "arch=compute_100a,code=sm_100a") == _build.ARCH


def test_host_only_entries_without_gpu():
    """Pure host arithmetic entries answer without a device."""
    L = _build.load()
    assert L.vt_comm_region_bytes(9, 1 << 20, 1 << 20, 1024) == 0       # > 8 ranks rejected
    a = L.vt_comm_region_bytes(2, 1 << 20, 64 << 20, 1 << 16)
    b = L.vt_comm_region_bytes(8, 1 << 20, 64 << 20, 1 << 16)
    assert a >= 2 * 2 * 2 * (1 << 20) and b >= 2 * 8 * 2 * (1 << 20)   # LL slots: parity x ranks x 2x data
    assert L.w8a8_gemv_ws_bytes(5, 5120) >= 256 + 5 * 5120 * 4
    assert L.vt_comm_create(0, 2, (ctypes.c_void_p * 2)(None, None), 1 << 20, 1 << 20, 1024) is None
