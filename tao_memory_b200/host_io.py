"""Decode-step operands in and results out through page-locked host memory.

The SMs move the bytes (``tao_copy_host_to_device`` / ``tao_copy_device_to_host``):
a kernel reads or writes the device-mapped page-locked buffer directly, so a
transfer of one decode step's tens of kilobytes costs about one round trip over the
host link instead of a copy engine's setup latency.  Both calls are asynchronous on
the current stream of the device tensor's device, like ``Tensor.copy_(...,
non_blocking=True)``.  No counterpart in the reference (its operands live on the
device already).
"""

import ctypes

import torch

from . import _lib


def _check(host, dev):
    if host.device.type != "cpu" or not host.is_pinned():
        raise ValueError("the host tensor must be page-locked (Tensor.pin_memory())")
    if dev.device.type != "cuda":
        raise ValueError("the device tensor must be a CUDA tensor")
    if not (host.is_contiguous() and dev.is_contiguous()):
        raise ValueError("host transfers need contiguous tensors")
    nbytes = host.numel() * host.element_size()
    if nbytes != dev.numel() * dev.element_size():
        raise ValueError("host and device tensors differ in size")
    return nbytes, torch.cuda.current_stream(dev.device).cuda_stream


def copy_to_device(dev, host):
    """dev <- host (page-locked); returns dev."""
    nbytes, stream = _check(host, dev)
    with torch.cuda.device(dev.device):
        _lib.check(_lib.lib().tao_copy_host_to_device(dev.data_ptr(), host.data_ptr(), nbytes, stream))
    return dev


def copy_to_host(host, dev):
    """host (page-locked) <- dev; returns host (valid once the stream has reached the copy)."""
    nbytes, stream = _check(host, dev)
    with torch.cuda.device(dev.device):
        _lib.check(_lib.lib().tao_copy_device_to_host(host.data_ptr(), dev.data_ptr(), nbytes, stream))
    return host


def copy_to_device_many(devs, hosts):
    """devs[i] <- hosts[i] (page-locked) for up to 8 pairs in one launch; returns devs.
    All device tensors must be on one device."""
    if not 0 < len(devs) == len(hosts) <= 8:
        raise ValueError("copy_to_device_many takes 1 to 8 (device, host) pairs")
    sizes = [_check(h, d)[0] for d, h in zip(devs, hosts)]
    device = devs[0].device
    if any(d.device != device for d in devs):
        raise ValueError("copy_to_device_many: device tensors on different devices")
    n = len(devs)
    dst = (ctypes.c_void_p * n)(*[d.data_ptr() for d in devs])
    src = (ctypes.c_void_p * n)(*[h.data_ptr() for h in hosts])
    nbytes = (ctypes.c_size_t * n)(*sizes)
    with torch.cuda.device(device):
        _lib.check(_lib.lib().tao_copy_host_to_device_many(dst, src, nbytes, n,
                                                           torch.cuda.current_stream(device).cuda_stream))
    return devs
