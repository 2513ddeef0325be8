"""Builds csrc/*.cu for sm_100a into vllm_turing_b200/libvllm_turing_b200.so and loads it with ctypes.

The reference compiles each csrc/<name>.cu with nvcc on first use and loads it through ctypes
(vllm_turing/_build.py:33-55); this package does the same for one library holding every kernel: one nvcc per source
(in parallel) into _build/*.o, one link, under a file lock. The library is rebuilt when the sha256 of its sources
differs from the stamp written next to it (not by mtime: a copied tree keeps the prebuilt library). There is no CPU
fallback: if the library cannot be built or loaded, every op raises.

Environment: VLLM_TURING_NVCC (nvcc path), VLLM_TURING_NO_BUILD=1 (never compile; a missing library is an error).
"""
import ctypes
import fcntl
import hashlib
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

_here = os.path.dirname(os.path.abspath(__file__))
_csrc = os.path.join(_here, "csrc")
_include = os.path.join(os.path.dirname(_here), "include")
LIB_NAME = "libvllm_turing_b200.so"
LIB_PATH = os.path.join(_here, LIB_NAME)
SOURCES = ("w8a8_gemv.cu", "w8a8_tc.cu", "gate_up_silu.cu", "w8a16_tc.cu", "norm_quant.cu", "ar8.cu", "tp_comm.cu",
           "tp_fused.cu", "tp_prefill.cu", "ref_abi.cu")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")
_lib = None


def _nvcc():
    for p in (os.environ.get("VLLM_TURING_NVCC"), "/usr/local/cuda/bin/nvcc"):
        if p and os.path.exists(p):
            return p
    raise RuntimeError("vllm_turing_b200: nvcc not found (set VLLM_TURING_NVCC)")


def _inputs():
    files = [os.path.join(_csrc, s) for s in SOURCES if os.path.exists(os.path.join(_csrc, s))]
    files += sorted(os.path.join(_csrc, f) for f in os.listdir(_csrc) if f.endswith((".cuh", ".h")))
    hdr = os.path.join(_include, "vllm_turing_b200.h")
    if os.path.exists(hdr):
        files.append(hdr)
    files.append(os.path.abspath(__file__))
    return files


def source_hash():
    h = hashlib.sha256()
    for f in _inputs():
        h.update(os.path.basename(f).encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def _stamp_path():
    return LIB_PATH + ".srchash"


def is_current():
    if not os.path.exists(LIB_PATH) or not os.path.exists(_stamp_path()):
        return False
    with open(_stamp_path()) as f:
        return f.read().strip() == source_hash()


def build(force=False, verbose=False):
    """Compile every CUDA source for sm_100a and link the library (no-op when current)."""
    os.makedirs(os.path.join(_here, "_build"), exist_ok=True)
    with open(os.path.join(_here, "_build", ".lock"), "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        if not force and is_current():
            return LIB_PATH
        nvcc = _nvcc()
        flags = ["-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC", "-I" + _csrc]
        if os.path.isdir(_include):
            flags += ["-I" + _include, "-DVT_HAVE_HEADER"]
        srcs = [s for s in SOURCES if os.path.exists(os.path.join(_csrc, s))]
        objs = [os.path.join(_here, "_build", s.replace(".cu", ".o")) for s in srcs]

        def cc(pair):
            src, obj = pair
            cmd = [nvcc, *flags, "-c", os.path.join(_csrc, src), "-o", obj]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"vllm_turing_b200: nvcc failed on {src}:\n{r.stderr[-4000:]}")
            if verbose and r.stderr:
                print(r.stderr)

        with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(cc, zip(srcs, objs)))
        tmp = LIB_PATH + ".tmp"
        r = subprocess.run([nvcc, "-shared", *ARCH, "-o", tmp, *objs], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"vllm_turing_b200: link failed:\n{r.stderr[-4000:]}")
        os.replace(tmp, LIB_PATH)
        with open(_stamp_path(), "w") as f:
            f.write(source_hash())
    return LIB_PATH


_P, _I, _LL, _SZ, _F, _U = (ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t, ctypes.c_float,
                            ctypes.c_uint)

# every export of include/vllm_turing_b200.h: name -> (restype, argtypes)
SIGNATURES = {
    "w8a8_gemv": (_I, [_P] * 6 + [_I] * 6 + [_P]),
    "w8a8_gemv_ws_bytes": (_SZ, [_I, _I]),
    "w8a8_gemv_ws": (_I, [_P] * 6 + [_I] * 6 + [_P, _SZ, _P]),
    "w8a8_gemv_noalloc": (_I, [_P] * 6 + [_I] * 6 + [_P]),
    "vt_gemv_s32": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "vt_status": (_U, [_I]),
    "vt_noalloc_status": (_U, [_I]),
    "vt_workspace_nonzero": (_LL, [_LL]),
    "w8a8_mma": (_I, [_P] * 6 + [_I] * 6 + [_P]),
    "w8a8_mma_ws_bytes": (_SZ, [_I, _I]),
    "w8a8_mma_ws": (_I, [_P] * 6 + [_I] * 6 + [_P, _SZ, _P]),
    "w8a8_mma_blocked_ws": (_I, [_P] * 6 + [_I] * 6 + [_P, _SZ, _P]),
    "w8a8_big": (_I, [_P] * 5 + [_I] * 4 + [_P]),
    "vt_gemm_s32": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "vt_gate_up_silu_quant_ws_bytes": (_SZ, [_I, _I]),
    "vt_gate_up_silu_quant": (_I, [_P] * 6 + [_I] * 5 + [_P, _SZ, _P]),
    "w8a16_gemv": (_I, [_P] * 5 + [_I] * 4 + [_P]),
    "w8a16_gemv_rows": (_I, [_P] * 5 + [_I] * 4 + [_P, _P]),
    "w8a16_mma": (_I, [_P] * 5 + [_I] * 4 + [_P]),
    "vt_w8a16_ws_bytes": (_SZ, [_I, _I]),
    "vt_w8a16_mm": (_I, [_P] * 5 + [_I] * 5 + [_P, _SZ, _P]),
    "vt_scaled_int8_quant": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "vt_rms_norm_quant": (_I, [_P, _P, _P, _F, _P, _P, _P, _I, _I, _I, _P]),
    "silu_mul_quant": (_I, [_P, _P, _P, _I, _I, _P]),
    "ar8_quant": (_I, [_P, _P, _I, _P]),
    "ar8_dequant_sum": (_I, [_P, _P, _I, _P]),
    "vt_ar8_dequant_sum": (_I, [_P, _P, _LL, _I, _P]),
    "vt_silu_mul_quant": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "ce_alloc": (_I, [_SZ, ctypes.POINTER(ctypes.c_void_p), _P]),
    "ce_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "ce_close": (_I, [_P]),
    "ce_free": (_I, [_P]),
    "ce_enable_peer": (_I, [_I]),
    "ce_driver_ok": (_I, []),
    "ce_all_reduce": (_I, [_P, _P, ctypes.c_long, _I, _P, _P, ctypes.c_long, _U, _I, _P]),
    "har_preload": (_I, []),
    "har_blocks": (_I, [_I]),
    "har_register": (_P, [_P, _SZ]),
    "har_unregister": (_I, [_P]),
    "har_all_reduce": (_I, [_P, _P, _I, _I, _P, _P, _P, _I, _P]),
    "dag_register": (_P, [_P, _SZ]),
    "dag_all_gather": (_I, [_P, _LL, _I, _P, _P, _P, _P, _I, _I] + [_P] * 6),
    "vt_set_wait_bounds": (_I, [ctypes.c_double, ctypes.c_double]),
    "vt_comm_region_bytes": (_SZ, [_I, _SZ, _SZ, _SZ]),
    "vt_comm_create": (_P, [_I, _I, ctypes.POINTER(ctypes.c_void_p), _SZ, _SZ, _SZ]),
    "vt_comm_destroy": (_I, [_P]),
    "vt_comm_ll_bytes": (_LL, [_P]),
    "vt_comm_big_bytes": (_LL, [_P]),
    "vt_comm_status": (_U, [_P, _I]),
    "vt_comm_seq": (_U, [_P]),
    "vt_all_reduce": (_I, [_P, _P, _P, _LL, _I, _I, _P]),
    "vt_all_gather": (_I, [_P, _P, _LL, _P]),
    "vt_comm_peer_copy": (_I, [_P, _I, _LL, _I, _I, _P]),
    "vt_all_gather_rows": (_I, [_P, _P, _LL, _LL, _LL, _P]),
    "vt_tp_row_linear": (_I, [_P] * 5 + [_P, _P, _F, _P, _P, _P] + [_I] * 4 + [_P]),
    "vt_tp_preload": (_I, []),
    "vt_tp_row_linear_prefill": (_I, [_P] * 5 + [_P, _P, _F, _P, _P, _P] + [_I] * 4 + [_P]),
    "vt_tp_prefill_preload": (_I, []),
}


def load():
    """The loaded library (built first if needed). Raises if it cannot be built or loaded: no CPU fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if os.environ.get("VLLM_TURING_NO_BUILD") == "1":
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"vllm_turing_b200: {LIB_PATH} missing and VLLM_TURING_NO_BUILD=1")
    elif not is_current():
        build()
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


lib = load
