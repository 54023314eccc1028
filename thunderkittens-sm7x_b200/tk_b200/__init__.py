"""Python binding of the tk_b200 C ABI (include/tk_b200.h).

The library is the product: ``libtk_b200.so`` built in-tree for sm_100a. This module
only loads it with ctypes and passes device pointers, sizes and CUDA streams. It
never computes anything itself and has no fallback: if the shared library is
missing, or a call returns an error, it raises.

Entry points mirror ThunderKittens-SM7x's public API (include/tk_sm7x/gemm.cuh,
attention.cuh, reduce.cuh, softmax.cuh): same argument meaning and the same
error behaviour (``cudaErrorInvalidValue`` for invalid arguments, nothing
enqueued).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libtk_b200.so")

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1
CUDA_ERROR_INVALID_DEVICE_FUNCTION = 98
CUDA_ERROR_NOT_SUPPORTED = 801

# Every symbol include/tk_b200.h declares, with its ctypes signature.
_VP, _I, _SZ, _F = C.c_void_p, C.c_int, C.c_size_t, C.c_float
SIGNATURES = {
    "tk_gemm_f16_f16_f32_nn": (_I, [_I, _I, _I, _VP, _I, _VP, _I, _VP, _I, _VP]),
    "tk_gemm_f16_f16_f32_nn_rowstats": (_I, [_I, _I, _I, _VP, _I, _VP, _I, _VP, _I, _VP, _VP, _VP]),
    "tk_gemm_f16_f16_f32_nn_rowstats_noalloc": (_I, [_I, _I, _I, _VP, _I, _VP, _I, _VP, _I, _VP, _VP,
                                                     _VP]),
    "tk_gemm_f16_f16_f32_nn_rowsoftmax": (_I, [_I, _I, _I, _VP, _I, _VP, _I, _VP, _I, _VP, _I, _VP]),
    "tk_gemm_f16_f16_f32_nn_gather": (_I, [_I, _I, _I, _VP, _I, _VP, _I, _VP, _I, _I, _I, _VP]),
    "tk_ipc_alloc": (_I, [_SZ, C.POINTER(C.c_void_p), _VP]),
    "tk_ipc_open": (_I, [_VP, C.POINTER(C.c_void_p)]),
    "tk_ipc_close": (_I, [_VP]),
    "tk_ipc_free": (_I, [_VP]),
    "tk_gemm_set_cta_group": (_I, [_I]),
    "tk_gemm_set_splitk_reduce": (_I, [_I]),
    "tk_tile_row_sum_f32": (_I, [_VP, _SZ, _VP, _VP]),
    "tk_tile_row_max_f32": (_I, [_VP, _SZ, _VP, _VP]),
    "tk_tile_row_softmax_f32": (_I, [_VP, _SZ, _VP, _VP]),
    "tk_tile_row_softmax_causal_f32": (_I, [_VP, _SZ, _VP, _VP]),
    "tk_tile_row_ops_f32": (_I, [_VP, _SZ, _VP, _VP, _VP, _VP, _VP]),
    "tk_attention_forward_16x16": (_I, [_VP, _VP, _VP, _VP, _VP]),
    "tk_attention_forward_16x16_causal": (_I, [_VP, _VP, _VP, _VP, _VP]),
    "tk_attention_forward_f16": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _F, _I, _VP]),
    "tk_attention_forward_gqa_f16": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _F, _I, _VP]),
    "tk_attention_set_cta_group": (_I, [_I]),
    "tk_gemm_set_group_rows": (_I, [_I]),
    "tk_gemm_set_small_m": (_I, [_I]),
    "tk_device_status": (_I, [C.POINTER(C.c_uint32), _I]),
    "tk_scratch_pool_bytes": (_I, [_I, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "tk_abi_version": (_I, []),
}

_lib = None


class TkError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} returned cudaError {code}")
        self.code = code


def build() -> None:
    """Compile libtk_b200.so for sm_100a (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-C", PKG_ROOT], check=True)


def lib():
    """The loaded C library. Raises if it was not built: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `make -C {PKG_ROOT}` (no CPU fallback exists)")
        handle = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _check(name: str, code: int) -> None:
    if code != CUDA_SUCCESS:
        raise TkError(name, code)


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ---- raw calls (pointers as ints or tensors); return the cudaError code -------------

def gemm_raw(m, n, k, a, lda, b, ldb, c, ldc, stream=None) -> int:
    return lib().tk_gemm_f16_f16_f32_nn(m, n, k, _ptr(a), lda, _ptr(b), ldb, _ptr(c), ldc, _stream(stream))


def gemm_rowstats_raw(m, n, k, a, lda, b, ldb, c, ldc, row_max, row_sum, stream=None) -> int:
    return lib().tk_gemm_f16_f16_f32_nn_rowstats(m, n, k, _ptr(a), lda, _ptr(b), ldb, _ptr(c), ldc,
                                                 _ptr(row_max), _ptr(row_sum), _stream(stream))


def gemm_rowsoftmax_raw(m, n, k, a, lda, b, ldb, c, ldc, probs, ldp, stream=None) -> int:
    return lib().tk_gemm_f16_f16_f32_nn_rowsoftmax(m, n, k, _ptr(a), lda, _ptr(b), ldb, _ptr(c), ldc,
                                                   _ptr(probs), ldp, _stream(stream))


def gemm_gather_raw(m, n, k, a, lda, b, ldb, c_ranks, rank, ldc, stream=None) -> int:
    """c_ranks: device pointers (ints) of every rank's gathered buffer, in rank order."""
    arr = (C.c_void_p * len(c_ranks))(*c_ranks)
    return lib().tk_gemm_f16_f16_f32_nn_gather(m, n, k, _ptr(a), lda, _ptr(b), ldb, C.cast(arr, C.c_void_p),
                                                len(c_ranks), rank, ldc, _stream(stream))


def ipc_alloc(nbytes: int) -> tuple[int, bytes]:
    """Shareable device allocation: (pointer, 64-byte IPC handle)."""
    ptr = C.c_void_p()
    handle = C.create_string_buffer(64)
    _check("tk_ipc_alloc", lib().tk_ipc_alloc(nbytes, C.byref(ptr), handle))
    return ptr.value, handle.raw


def ipc_open(handle: bytes) -> int:
    ptr = C.c_void_p()
    buf = C.create_string_buffer(bytes(handle), 64)
    _check("tk_ipc_open", lib().tk_ipc_open(buf, C.byref(ptr)))
    return ptr.value


def ipc_close(ptr: int) -> None:
    _check("tk_ipc_close", lib().tk_ipc_close(ptr))


def ipc_free(ptr: int) -> None:
    _check("tk_ipc_free", lib().tk_ipc_free(ptr))


def set_gemm_cta_group(g: int) -> int:
    return lib().tk_gemm_set_cta_group(g)


def set_gemm_splitk_reduce(mode: int) -> int:
    """0: split-K partials summed inside the kernel (tile clusters) where they fit;
    1: always by a second kernel. Returns the previous mode."""
    return lib().tk_gemm_set_splitk_reduce(mode)


def attention_16x16_raw(q, k, v, out, causal=False, stream=None) -> int:
    fn = lib().tk_attention_forward_16x16_causal if causal else lib().tk_attention_forward_16x16
    return fn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _stream(stream))


def attention_raw(q, k, v, out, batch, heads, seq, head_dim, scale, causal, stream=None) -> int:
    return lib().tk_attention_forward_f16(_ptr(q), _ptr(k), _ptr(v), _ptr(out), batch, heads, seq,
                                          head_dim, float(scale), 1 if causal else 0, _stream(stream))


def attention_gqa_raw(q, k, v, out, batch, heads_q, heads_kv, seq, head_dim, scale, causal, stream=None) -> int:
    return lib().tk_attention_forward_gqa_f16(_ptr(q), _ptr(k), _ptr(v), _ptr(out), batch, heads_q, heads_kv,
                                              seq, head_dim, float(scale), 1 if causal else 0, _stream(stream))


def row_ops_raw(tiles, n_tiles, row_sum=None, row_max=None, softmax=None, softmax_causal=None,
                stream=None) -> int:
    return lib().tk_tile_row_ops_f32(_ptr(tiles), n_tiles, _ptr(row_sum), _ptr(row_max), _ptr(softmax),
                                     _ptr(softmax_causal), _stream(stream))


def device_status(clear: bool = False) -> int:
    v = C.c_uint32()
    _check("tk_device_status", lib().tk_device_status(C.byref(v), 1 if clear else 0))
    return v.value


def scratch_pool_bytes(device: int = 0) -> tuple[int, int]:
    """(reserved, used) bytes of the library's scratch pool on `device`."""
    reserved, used = C.c_uint64(), C.c_uint64()
    _check("tk_scratch_pool_bytes", lib().tk_scratch_pool_bytes(device, C.byref(reserved), C.byref(used)))
    return reserved.value, used.value


# ---- torch-level helpers (device tensors in, device tensors out) ---------------------

def gemm(a, b, c=None, *, m=None, n=None, k=None, lda=None, ldb=None, ldc=None, stream=None):
    """C = A @ B with A (m x lda) / B (k x ldb) binary16 and C (m x ldc) FP32 device tensors."""
    import torch
    m = a.shape[0] if m is None else m
    k = b.shape[0] if k is None else k
    n = b.shape[1] if n is None else n
    lda = a.stride(0) if lda is None else lda
    ldb = b.stride(0) if ldb is None else ldb
    if c is None:
        c = torch.empty((m, n), dtype=torch.float32, device=a.device)
    ldc = c.stride(0) if ldc is None else ldc
    _check("tk_gemm_f16_f16_f32_nn", gemm_raw(m, n, k, a, lda, b, ldb, c, ldc, stream))
    return c


def gemm_rowstats(a, b, c=None, *, stream=None):
    import torch
    m, n, k = a.shape[0], b.shape[1], b.shape[0]
    if c is None:
        c = torch.empty((m, n), dtype=torch.float32, device=a.device)
    row_max = torch.empty(m, dtype=torch.float32, device=a.device)
    row_sum = torch.empty(m, dtype=torch.float32, device=a.device)
    _check("tk_gemm_f16_f16_f32_nn_rowstats",
           gemm_rowstats_raw(m, n, k, a, a.stride(0), b, b.stride(0), c, c.stride(0), row_max, row_sum,
                             stream))
    return c, row_max, row_sum


def gemm_rowsoftmax(a, b, c=None, probs=None, *, in_place=False, stream=None):
    """C = A @ B and P = softmax over each row of C. With in_place=True P replaces C
    (one buffer); returns (C, P), the same tensor twice when in place."""
    import torch
    m, n, k = a.shape[0], b.shape[1], b.shape[0]
    if c is None:
        c = torch.empty((m, n), dtype=torch.float32, device=a.device)
    if in_place:
        probs = c
    elif probs is None:
        probs = torch.empty((m, n), dtype=torch.float32, device=a.device)
    _check("tk_gemm_f16_f16_f32_nn_rowsoftmax",
           gemm_rowsoftmax_raw(m, n, k, a, a.stride(0), b, b.stride(0), c, c.stride(0), probs,
                               probs.stride(0), stream))
    return c, probs


def tile_row_ops(tiles, *, ops=("sum", "max", "softmax", "causal"), stream=None):
    """Batched 16x16 tile row ops; tiles is a contiguous FP32 tensor of n*256 values."""
    import torch
    n = tiles.numel() // 256
    out = {}
    dev = tiles.device
    if "sum" in ops:
        out["sum"] = torch.empty((n, 16), dtype=torch.float32, device=dev)
    if "max" in ops:
        out["max"] = torch.empty((n, 16), dtype=torch.float32, device=dev)
    if "softmax" in ops:
        out["softmax"] = torch.empty((n, 16, 16), dtype=torch.float32, device=dev)
    if "causal" in ops:
        out["causal"] = torch.empty((n, 16, 16), dtype=torch.float32, device=dev)
    _check("tk_tile_row_ops_f32", row_ops_raw(tiles, n, out.get("sum"), out.get("max"), out.get("softmax"),
                                              out.get("causal"), stream))
    return out


def attention(q, k, v, *, scale, causal=False, out=None, stream=None):
    """q, k, v: [B, H, S, D] contiguous binary16 device tensors -> FP32 [B, H, S, D]."""
    import torch
    b, h, s, d = q.shape
    if out is None:
        out = torch.empty((b, h, s, d), dtype=torch.float32, device=q.device)
    _check("tk_attention_forward_f16", attention_raw(q, k, v, out, b, h, s, d, scale, causal, stream))
    return out
