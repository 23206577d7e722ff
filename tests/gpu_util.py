"""Small raw-memory helpers for the GPU tests (device addresses that are not
torch tensors, e.g. PagedKVStorage.key_base()), via the CUDA runtime that
torch has already loaded."""
import ctypes

import numpy as np
import torch

_rt = None


def cudart():
    global _rt
    if _rt is None:
        torch.cuda.init()
        _rt = ctypes.CDLL("libcudart.so.12")
        _rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        _rt.cudaMemset.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t]
    return _rt


def d2h(addr: int, nbytes: int) -> np.ndarray:
    torch.cuda.synchronize()
    out = np.empty(nbytes, np.uint8)
    assert cudart().cudaMemcpy(out.ctypes.data, addr, nbytes, 2) == 0
    return out


def h2d(addr: int, data: np.ndarray) -> None:
    data = np.ascontiguousarray(data)
    torch.cuda.synchronize()
    assert cudart().cudaMemcpy(addr, data.ctypes.data, data.nbytes, 1) == 0


def memset(addr: int, value: int, nbytes: int) -> None:
    torch.cuda.synchronize()
    assert cudart().cudaMemset(addr, value, nbytes) == 0
    torch.cuda.synchronize()


def read_elem(addr: int, elem: int) -> int:
    raw = d2h(addr, elem)
    return int(raw.view(np.uint16 if elem == 2 else np.uint32)[0])
