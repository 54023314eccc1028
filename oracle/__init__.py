"""CPU oracle for the ThunderKittens-SM7x hot path (test infrastructure only).

This package is the checker. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import it; the CUDA library never does, and it
raises instead of falling back to anything here.

``lib()`` loads ``oracle/_build/libtk_oracle.so``: a plain C++ restatement of the
reference's host oracles (see ``tk_oracle.h`` for the file:line each follows).
``ref_lib()`` loads ``oracle/_ref/libtk_ref.so`` when present: the reference's own
host oracle functions compiled from its sources by ``make -C oracle ref``. The
golden fixtures in ``tests/golden/`` were produced from that library.
``legacy_lib()`` loads ``oracle/_ref/libtk_legacy.so`` when present: the reference's
own GEMM and attention kernels built as compute_75 PTX (``make -C oracle legacy``),
which the driver JIT-compiles for the GPU at hand. It is the legacy-path comparison
datapoint: it runs the reference's SM7x code on the same device, never the product.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libtk_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtk_ref.so")
LEGACY_SO = os.path.join(HERE, "_ref", "libtk_legacy.so")

_lock = threading.Lock()
_lib = None
_ref = None
_legacy = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")


def ref_root() -> str:
    """The ThunderKittens-SM7x source tree: $REF_ROOT, else a `reference` directory
    beside this repository's checkout (it is only read by the `ref` and `legacy`
    build recipes, never at test or bench time)."""
    return os.environ.get("REF_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def build(ref: bool = False) -> None:
    """Compile the oracle (and, if asked and the reference tree exists, _ref)."""
    targets = ["all"]
    root = ref_root()
    if ref and os.path.isdir(root):
        targets += ["ref", "legacy", f"REF_ROOT={root}"]
    subprocess.run(["make", "-s", "-C", HERE, *targets], check=True)


def _declare(lib):
    sig = {
        "tko_f32_to_f16": (C.c_uint16, [C.c_float]),
        "tko_f64_to_f16": (C.c_uint16, [C.c_double]),
        "tko_f16_to_f32": (C.c_float, [C.c_uint16]),
        "tko_f32_to_f16_array": (None, [_f32p, _u16p, C.c_size_t]),
        "tko_f16_to_f32_array": (None, [_u16p, _f32p, C.c_size_t]),
        "tko_gen_gemm_uniform": (None, [C.c_uint32, C.c_float, C.c_float, C.c_int, C.c_int, C.c_int,
                                        _u16p, C.c_int, _u16p, C.c_int]),
        "tko_gen_gemm_normal": (None, [C.c_uint32, C.c_float, C.c_int, C.c_int, C.c_int,
                                       _u16p, C.c_int, _u16p, C.c_int]),
        "tko_gen_normal_f32": (None, [C.c_uint32, C.c_float, _f32p, C.c_size_t]),
        "tko_gen_qkv_normal": (None, [C.c_uint32, C.c_float, C.c_size_t, _u16p, _u16p, _u16p]),
        "tko_gemm_ref_f64": (None, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                    C.c_int, C.c_void_p, C.c_void_p, C.c_int]),
        "tko_error_bound": (C.c_double, [C.c_int, C.c_double]),
        "tko_error_bound_extended": (C.c_double, [C.c_int, C.c_double]),
        "tko_within_bound": (C.c_int, [C.c_double, C.c_double, C.c_double]),
        "tko_gemm_check": (C.c_size_t, [C.c_int, C.c_int, C.c_int, _f32p, C.c_int, _f64p, _f64p,
                                        C.c_int, C.c_uint32, C.c_int, C.POINTER(C.c_double),
                                        C.POINTER(C.c_double)]),
        "tko_row_tree16": (C.c_float, [_f32p, C.c_int]),
        "tko_tile_row_reduce": (None, [_f32p, C.c_size_t, _f32p, C.c_int]),
        "tko_pairwise_reduce": (C.c_float, [_f32p, C.c_size_t, C.c_size_t, C.c_int]),
        "tko_matrix_row_stats": (None, [_f32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]),
        "tko_tile_row_softmax_f64": (None, [_f32p, C.c_size_t, _f64p, C.c_int]),
        "tko_tile_row_softmax_check": (C.c_size_t, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                                    C.c_double, C.POINTER(C.c_double)]),
        "tko_row_softmax_check": (C.c_size_t, [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p,
                                               C.c_size_t, C.c_double, C.POINTER(C.c_double)]),
        "tko_attention_ref_f64": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                         C.c_double, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                         C.c_void_p]),
        "tko_attention_bound": (None, [_u16p, C.c_int, C.c_int, _f64p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(ORACLE_SO):
                build()
            handle = C.CDLL(ORACLE_SO)
            _declare(handle)
            _lib = handle
        return _lib


def ref_lib():
    """The reference's own host oracles, or None when oracle/_ref was not built."""
    global _ref
    with _lock:
        if _ref is None and os.path.exists(REF_SO):
            _ref = C.CDLL(REF_SO)
            _ref.tkref_error_bound.restype = C.c_double
            _ref.tkref_error_bound.argtypes = [C.c_int, C.c_double]
            _ref.tkref_within_bound.restype = C.c_int
            _ref.tkref_within_bound.argtypes = [C.c_double, C.c_double, C.c_double]
            _ref.tkref_canonical_row.restype = C.c_float
            _ref.tkref_canonical_row.argtypes = [_f32p, C.c_int]
            _ref.tkref_rounding_census.restype = C.c_int
            _ref.tkref_rounding_census.argtypes = [_f32p]
            _ref.tkref_row_exact_value.restype = C.c_uint16
            _ref.tkref_row_exact_value.argtypes = [C.c_int, C.c_int, C.c_int]
            _ref.tkref_row_rounded_value.restype = C.c_uint16
            _ref.tkref_row_rounded_value.argtypes = [C.c_int, C.c_int, C.c_uint32]
            _ref.tkref_softmax_logit.restype = C.c_float
            _ref.tkref_softmax_logit.argtypes = [C.c_int] * 4
            _ref.tkref_causal_logit.restype = C.c_double
            _ref.tkref_causal_logit.argtypes = [C.c_int] * 3
            _ref.tkref_midpoint_margin.restype = C.c_double
            _ref.tkref_midpoint_margin.argtypes = [C.c_double, C.c_uint16]
            _ref.tkref_diff_model_case.restype = C.c_char_p
            _ref.tkref_diff_model_case.argtypes = [C.c_int, C.POINTER(C.c_int)]
            _ref.tkref_corr_sentinel.restype = C.c_float
        return _ref


def legacy_lib():
    """The reference's GEMM / attention kernels as JIT-compiled PTX (the legacy SM7x
    path on the current device), or None when oracle/_ref was not built."""
    global _legacy
    with _lock:
        if _legacy is None and os.path.exists(LEGACY_SO):
            handle = C.CDLL(LEGACY_SO)
            handle.tkl_gemm_f16_f16_f32_nn.restype = C.c_int
            handle.tkl_gemm_f16_f16_f32_nn.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                                       C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]
            handle.tkl_attention_forward_16x16.restype = C.c_int
            handle.tkl_attention_forward_16x16.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_void_p]
            _legacy = handle
        return _legacy


def _ptr(arr: np.ndarray):
    assert arr.flags["C_CONTIGUOUS"]
    return arr.ctypes.data_as(C.c_void_p)


# ---- numpy-level helpers --------------------------------------------------------

def f32_to_f16_bits(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().tko_f32_to_f16_array(x.reshape(-1), out.reshape(-1), x.size)
    return out


def f16_bits_to_f32(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().tko_f16_to_f32_array(h.reshape(-1), out.reshape(-1), h.size)
    return out


def gen_gemm_uniform(seed, m, n, k, lda, ldb, lo=-1.0, hi=1.0, pad_bits=0):
    a = np.full((m, lda), pad_bits, dtype=np.uint16)
    b = np.full((k, ldb), pad_bits, dtype=np.uint16)
    lib().tko_gen_gemm_uniform(seed, lo, hi, m, n, k, a.reshape(-1), lda, b.reshape(-1), ldb)
    return a, b


def gen_gemm_normal(seed, sigma, m, n, k, lda, ldb, pad_bits=0):
    a = np.full((m, lda), pad_bits, dtype=np.uint16)
    b = np.full((k, ldb), pad_bits, dtype=np.uint16)
    lib().tko_gen_gemm_normal(seed, sigma, m, n, k, a.reshape(-1), lda, b.reshape(-1), ldb)
    return a, b


def gen_normal_f32(seed, sigma, count) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().tko_gen_normal_f32(seed, sigma, out, count)
    return out


def gen_qkv_normal(seed, sigma, count):
    q = np.empty(count, dtype=np.uint16)
    k = np.empty(count, dtype=np.uint16)
    v = np.empty(count, dtype=np.uint16)
    lib().tko_gen_qkv_normal(seed, sigma, count, q, k, v)
    return q, k, v


def gemm_ref(m, n, k, a, lda, b, ldb, row_begin=0, row_end=None):
    """FP64 R and S for rows [row_begin, row_end) (tests/gemm_differential.cu:380-401)."""
    if row_end is None:
        row_end = m
    rows = row_end - row_begin
    a = np.ascontiguousarray(a, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    r = np.empty((rows, n), dtype=np.float64)
    s = np.empty((rows, n), dtype=np.float64)
    a_off = a.reshape(-1)[row_begin * lda:]
    lib().tko_gemm_ref_f64(rows, n, k, _ptr(a_off), lda, _ptr(b.reshape(-1)), ldb, _ptr(r), _ptr(s), n)
    return r, s


def gemm_check(k, c, r, s, n, ldc, sentinel_bits=0, check_padding=False):
    """Counts cells outside the (extended) GEMM bound; returns (failures, max_abs, max_ratio)."""
    c = np.ascontiguousarray(c, dtype=np.float32)
    m = r.shape[0]
    ma, mr = C.c_double(), C.c_double()
    fails = lib().tko_gemm_check(m, n, k, c.reshape(-1), ldc, np.ascontiguousarray(r).reshape(-1),
                                 np.ascontiguousarray(s).reshape(-1), r.shape[1], sentinel_bits,
                                 1 if check_padding else 0, C.byref(ma), C.byref(mr))
    return int(fails), ma.value, mr.value


def error_bound(k, s):
    return lib().tko_error_bound(k, s)


def error_bound_extended(k, s):
    return lib().tko_error_bound_extended(k, s)


def tile_row_reduce(tiles, op: str) -> np.ndarray:
    t = np.ascontiguousarray(tiles, dtype=np.float32).reshape(-1)
    n = t.size // 256
    out = np.empty(n * 16, dtype=np.float32)
    lib().tko_tile_row_reduce(t, n, out, 0 if op == "sum" else 1)
    return out.reshape(n, 16)


def pairwise_reduce(x, op: str) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    return lib().tko_pairwise_reduce(x, x.size, 1, 0 if op == "sum" else 1)


def matrix_row_stats(c, m, n, ldc):
    c = np.ascontiguousarray(c, dtype=np.float32).reshape(-1)
    mx = np.empty(m, dtype=np.float32)
    sm = np.empty(m, dtype=np.float32)
    lib().tko_matrix_row_stats(c, m, n, ldc, mx, sm)
    return mx, sm


def tile_row_softmax_f64(tiles, causal: bool) -> np.ndarray:
    t = np.ascontiguousarray(tiles, dtype=np.float32).reshape(-1)
    n = t.size // 256
    out = np.empty(n * 256, dtype=np.float64)
    lib().tko_tile_row_softmax_f64(t, n, out, 1 if causal else 0)
    return out.reshape(n, 16, 16)


SOFTMAX_BOUND = 512.0 * 2.0 ** -23  # tests/tile_softmax.cu:20


def tile_row_softmax_check(tiles, got, causal: bool, bound: float = SOFTMAX_BOUND):
    t = np.ascontiguousarray(tiles, dtype=np.float32).reshape(-1)
    g = np.ascontiguousarray(got, dtype=np.float32).reshape(-1)
    assert t.size == g.size
    err = C.c_double()
    fails = lib().tko_tile_row_softmax_check(_ptr(t), _ptr(g), t.size // 256, 1 if causal else 0,
                                             bound, C.byref(err))
    return int(fails), err.value


def row_softmax_check(x, got, bound: float = SOFTMAX_BOUND):
    """Full-row softmax of the 2-D FP32 array x against `got` (same shape): returns
    (failures, max_abs_error)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    g = np.ascontiguousarray(got, dtype=np.float32)
    assert x.shape == g.shape and x.ndim == 2
    err = C.c_double()
    fails = lib().tko_row_softmax_check(_ptr(x), x.shape[0], x.shape[1], x.shape[1], _ptr(g), g.shape[1],
                                        bound, C.byref(err))
    return int(fails), err.value


def attention_ref(q, k, v, s, d, scale, causal, row_begin=0, row_end=None, want_prob=False):
    """FP64 attention of one (batch, head) slice with FP16-rounded normalised P."""
    if row_end is None:
        row_end = s
    q = np.ascontiguousarray(q, dtype=np.uint16).reshape(-1)
    k = np.ascontiguousarray(k, dtype=np.uint16).reshape(-1)
    v = np.ascontiguousarray(v, dtype=np.uint16).reshape(-1)
    rows = row_end - row_begin
    out = np.empty((rows, d), dtype=np.float64)
    prob = np.empty((rows, s), dtype=np.float64) if want_prob else None
    lib().tko_attention_ref_f64(_ptr(q), _ptr(k), _ptr(v), s, d, float(scale), 1 if causal else 0,
                                row_begin, row_end, _ptr(out), _ptr(prob) if want_prob else None)
    return (out, prob) if want_prob else out


def attention_bound(v, s, d) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.uint16).reshape(-1)
    out = np.empty(d, dtype=np.float64)
    lib().tko_attention_bound(v, s, d, out)
    return out
