"""ctypes binding of libnufft_b200.so (the C ABI declared in include/nufft_b200.h).

Loading is strict: if the shared library is missing the import fails with an
explicit error -- there is no CPU or pure-Python fallback for any transform.
Build it with ``python mlx_nufft_b200/build.py``.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# NUFFT_B200_LIB names an alternate build of the same library (a tuning
# build from `build.py --out PATH -DNAME=VALUE`); default: the in-tree one.
LIB_PATH = os.environ.get("NUFFT_B200_LIB") or os.path.join(_HERE, "libnufft_b200.so")

NUFFT_OK = 0
NUFFT_ERR_ARG = -1
NUFFT_ERR_OOM = -2
NUFFT_ERR_CUDA = -3
NUFFT_ERR_CUFFT = -4
NUFFT_ERR_STATE = -5
NUFFT_ERR_RANGE = -6
NUFFT_ERR_UNSUPPORTED = -7

PREC = {"crit64": 0, "fp32": 1, "coords64": 2, "phases64": 3}
METHOD = {"auto": 0, "od": 1, "tiled": 1, "gm": 2, "global": 2}
STAGE_ALL, STAGE_SPREAD, STAGE_FINISH = 0, 1, 2   # type 2: grid, interp

c_double_p = ctypes.POINTER(ctypes.c_double)
c_int64_p = ctypes.POINTER(ctypes.c_int64)


class NufftOpts(ctypes.Structure):
    _fields_ = [
        ("upsampfac", ctypes.c_double),
        ("sigma_inner", ctypes.c_double),
        ("prec", ctypes.c_int),
        ("method", ctypes.c_int),
        ("sort_points", ctypes.c_int),
        ("max_batch", ctypes.c_int),
        ("profile", ctypes.c_int),
        ("has_source_extent", ctypes.c_int),
        ("source_extent", ctypes.c_double * 6),
        ("kerevalmeth", ctypes.c_int),
        ("fft_prec", ctypes.c_int),
    ]


class NufftPlanInfo(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int), ("dim", ctypes.c_int),
        ("n_trans", ctypes.c_int), ("isign", ctypes.c_int),
        ("w", ctypes.c_int), ("w2", ctypes.c_int),
        ("beta", ctypes.c_double), ("beta2", ctypes.c_double),
        ("eps", ctypes.c_double), ("upsampfac", ctypes.c_double),
        ("sigma_inner", ctypes.c_double),
        ("n_modes", ctypes.c_int64 * 3),
        ("nf", ctypes.c_int64 * 3),
        ("n_up", ctypes.c_int64 * 3),
        ("M", ctypes.c_int64),
        ("N_tgt", ctypes.c_int64),
        ("C", ctypes.c_double * 3),
        ("D", ctypes.c_double * 3),
        ("gam", ctypes.c_double * 3),
        ("tiled", ctypes.c_int),
        ("bin", ctypes.c_int * 3),
        ("nsub", ctypes.c_int64),
        ("nsub_tgt", ctypes.c_int64),
        ("device_bytes", ctypes.c_int64),
        ("kernel_launches", ctypes.c_int64),
        ("fft_execs", ctypes.c_int64),
        ("fft64", ctypes.c_int),
        ("fft_own", ctypes.c_int),
        ("grid_cells", ctypes.c_int64),
        ("grid_ext", ctypes.c_int64 * 3),
        ("grid_lo", ctypes.c_int * 3),
    ]


# name -> (restype, argtypes)
_PROTOS = {
    "nufft_default_opts": (None, [ctypes.POINTER(NufftOpts)]),
    "nufft_plan_create": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int, c_int64_p, ctypes.c_int, ctypes.c_double,
        ctypes.c_int, ctypes.POINTER(NufftOpts), ctypes.c_int,
        ctypes.POINTER(ctypes.c_void_p)]),
    "nufft_setpts": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p]),
    "nufft_set_sources": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p]),
    "nufft_execute": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ctypes.c_void_p]),
    "nufft_execute_adjoint": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ctypes.c_void_p]),
    "nufft_execute_stage": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_void_p]),
    "nufft_get_grid": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), c_int64_p]),
    "nufft_execute_disjoint": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p]),
    "nufft_plan_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "nufft_plan_check": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "nufft_plan_get_info": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(NufftPlanInfo)]),
    "nufft_get_stage_times": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int]),
    "nufft_plan_set_profile": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "nufft_debug_points": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p]),
    "nufft_expi": (ctypes.c_int, [
        ctypes.c_int, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int64,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "nufft_interp_noalloc": (ctypes.c_int, [
        ctypes.c_int, c_int64_p, ctypes.c_double, ctypes.c_double,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "nufft_kernel_params": (ctypes.c_int, [
        ctypes.c_double, ctypes.c_double, ctypes.POINTER(ctypes.c_int),
        c_double_p]),
    "nufft_next235even": (ctypes.c_int64, [ctypes.c_int64]),
    "nufft_kernel_ft": (ctypes.c_int, [
        ctypes.c_int64, c_double_p, ctypes.c_double, ctypes.c_int,
        c_double_p]),
    "nufft_set_nhg_type3": (ctypes.c_int, [
        ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_int,
        c_int64_p, c_double_p, c_double_p]),
    "nufft_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int]),
    "nufft_version": (ctypes.c_char_p, []),
    "nufft_device_count": (ctypes.c_int, []),
}

EXPORTED = tuple(_PROTOS)


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"mlx_nufft_b200: native library {LIB_PATH} is missing; build it "
            "with `python mlx_nufft_b200/build.py` (nvcc, sm_100a). There is "
            "no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _PROTOS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error():
    buf = ctypes.create_string_buffer(1024)
    lib.nufft_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc, what=""):
    """Raise the Python exception matching a C status code."""
    if rc >= 0:
        return rc
    msg = last_error() or what
    if rc in (NUFFT_ERR_ARG, NUFFT_ERR_RANGE):
        raise ValueError(msg)
    if rc == NUFFT_ERR_STATE:
        raise RuntimeError(msg)
    if rc == NUFFT_ERR_OOM:
        raise MemoryError(msg)
    if rc == NUFFT_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"{msg} (status {rc})")


def default_opts():
    o = NufftOpts()
    lib.nufft_default_opts(ctypes.byref(o))
    return o
