"""Helpers shared by setup, the codec and the GPU export.

Same contracts as neuralzip/utils.py:1-115 (named-tensor walks, raw byte
views, exponent histograms, the base-2 Jensen-Shannon distance, the
per-stream chunk size and a perf_counter timer).
"""

import math
import time
from collections.abc import Mapping
from itertools import chain

import numpy as np
import torch

from neuralzip_b200.dtypes import DTYPES


def _named_tensors(value, prefix=""):
    if torch.is_tensor(value):
        yield prefix, value
    elif isinstance(value, Mapping):
        for key, child in value.items():
            yield from _named_tensors(child, str(key) if not prefix else f"{prefix}.{key}")
    elif isinstance(value, (list, tuple)):
        for index, child in enumerate(value):
            yield from _named_tensors(child, str(index) if not prefix else f"{prefix}.{index}")


def _model_tensors(model):
    if isinstance(model, Mapping):
        items = _named_tensors(model)
    elif isinstance(model, torch.nn.Module):
        persistent = set(model.state_dict())
        items = chain(model.named_parameters(),
                      ((n, t) for n, t in model.named_buffers() if n in persistent))
    else:
        raise TypeError("Expected a tensor mapping or torch.nn.Module.")
    tensors = [(str(n), t) for n, t in items if torch.is_tensor(t) and t.is_floating_point()]
    if not tensors:
        raise ValueError("No floating tensors were found.")
    if len({n for n, _ in tensors}) != len(tensors):
        raise ValueError("Tensor names must be unique.")
    return tensors


def _floating_tensors(named_tensors):
    for name, tensor in sorted(named_tensors, key=lambda item: item[0]):
        if torch.is_tensor(tensor) and tensor.is_floating_point() and tensor.numel():
            yield name, tensor


def _tensor_raw_bytes(tensor):
    tensor = tensor.detach().cpu().contiguous()
    return tensor.reshape(-1).view(torch.uint8).numpy().tobytes()


def _tensor_from_raw_bytes(raw_bytes, dtype, shape):
    owner = raw_bytes if isinstance(raw_bytes, bytearray) else bytearray(raw_bytes)
    shape = tuple(int(d) for d in shape)
    expected = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
    if len(owner) != expected:
        raise ValueError(f"Decoded tensor byte length mismatch: {len(owner)} != {expected}.")
    if not owner:
        return torch.empty(shape, dtype=dtype)
    return torch.frombuffer(owner, dtype=torch.uint8).view(dtype).reshape(shape)


def exponent_distribution(tensor):
    """Normalized exponent histogram of a floating tensor."""
    config = DTYPES[tensor.dtype]
    exponent = config.extract_exponents(_tensor_raw_bytes(tensor))
    counts = np.bincount(exponent, minlength=256).astype(np.float64)
    total = counts.sum()
    return counts / total if total else counts


def jensen_shannon_distance(left, right):
    """Base-2 Jensen-Shannon distance between two distributions."""
    left = np.asarray(left, dtype=np.float64)
    right = np.asarray(right, dtype=np.float64)
    middle = 0.5 * (left + right)
    lm, rm = left > 0, right > 0
    divergence = 0.5 * np.sum(left[lm] * np.log2(left[lm] / middle[lm]))
    divergence += 0.5 * np.sum(right[rm] * np.log2(right[rm] / middle[rm]))
    return float(np.sqrt(max(float(divergence), 0.0)))


def _stream_chunk_size(chunk_size, element_size):
    return max(1, chunk_size // int(element_size))


def time_call(func, /, *args, **kwargs):
    """Call a function and return the result and elapsed seconds."""
    start = time.perf_counter()
    return func(*args, **kwargs), time.perf_counter() - start
