"""Small GPU-test helpers: numpy <-> device tensors and the CUDA runtime's
pending-error API (the same libcudart the library uses), for the reference's
"stale error" contract checks (tests/gemm_correctness.cu:217-224, 252-314)."""

import ctypes as C

import numpy as np
import torch

_rt = None


def cudart():
    global _rt
    if _rt is None:
        torch.cuda.init()
        _rt = C.CDLL("libcudart.so.12")
        _rt.cudaGetLastError.restype = C.c_int
        _rt.cudaPeekAtLastError.restype = C.c_int
        _rt.cudaSetDevice.restype = C.c_int
        _rt.cudaSetDevice.argtypes = [C.c_int]
        _rt.cudaGetDevice.restype = C.c_int
        _rt.cudaGetDevice.argtypes = [C.POINTER(C.c_int)]
    return _rt


def seed_stale_error() -> int:
    """Leave a non-sticky error pending on this thread (an invalid device ordinal)."""
    rt = cudart()
    cur = C.c_int()
    assert rt.cudaGetDevice(C.byref(cur)) == 0
    code = rt.cudaSetDevice(1 << 20)
    assert code != 0
    assert rt.cudaPeekAtLastError() == code
    return code


def dev(arr: np.ndarray) -> torch.Tensor:
    """Copies a numpy array to cuda:0 (uint16 arrays become binary16 tensors)."""
    a = np.ascontiguousarray(arr)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.float16).cuda()
    return torch.from_numpy(a.copy()).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    if t.dtype == torch.float16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    return t.cpu().numpy()
