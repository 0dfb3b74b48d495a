"""Helpers shared by the GPU tests: numpy <-> device tensors and ctypes
pointers for calling libaeth_galore through its C ABI."""
import ctypes as C

import numpy as np
import torch

DEV = "cuda:0"


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def bf16_dev_from_bits(bits):
    """uint16 bf16 bit patterns -> a bfloat16 device tensor."""
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV)
    return t.view(torch.bfloat16)


def rel_fro(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm((a - b).ravel())
    n = np.linalg.norm(b.ravel())
    return d / n if n > 0 else d
