"""Helpers for the GPU parity tests: torch is used only as device-memory and
stream plumbing; every computation under test goes through libarcllm_cuda.so."""
import ctypes as C

import numpy as np
import torch

import arcllm_b200 as A


def dev():
    return torch.device("cuda:0")


def to_dev(a):
    """numpy array -> contiguous CUDA tensor with the same bytes."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(dev())


def empty_f32(n):
    return torch.empty(n, dtype=torch.float32, device=dev())


def empty_u8(n):
    return torch.empty(n, dtype=torch.uint8, device=dev())


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def check_device_error():
    bits = C.c_uint32(0)
    A.call("arcllm_cuda_device_error", stream(), C.byref(bits))
    assert bits.value == 0, "device error word = %#x" % bits.value
