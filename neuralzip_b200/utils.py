"""Small helpers shared by setup, the storage codec and the GPU export.

``_model_tensors`` follows the naming of neuralzip/utils.py:12-50 (dotted
paths through nested mappings and sequences; a module's parameters and
persistent buffers under their state-dict names), since setup keys and
checkpoint tensor names are built from it.
"""

import time
from collections.abc import Mapping

import torch


def _tensor_items(value):
    """(dotted name, tensor) for every tensor inside nested mappings, lists
    and tuples, depth first, in insertion order."""
    stack = [("", value)]
    while stack:
        prefix, node = stack.pop()
        if torch.is_tensor(node):
            yield prefix, node
            continue
        if isinstance(node, Mapping):
            children = [(str(key), child) for key, child in node.items()]
        elif isinstance(node, (list, tuple)):
            children = [(str(index), child) for index, child in enumerate(node)]
        else:
            continue
        stack.extend((f"{prefix}.{key}" if prefix else key, child) for key, child in reversed(children))


def _model_tensors(model):
    """Named floating tensors of a model (parameters and persistent buffers)
    or of a nested tensor mapping; names must be unique."""
    if isinstance(model, torch.nn.Module):
        persistent = set(model.state_dict())
        items = list(model.named_parameters())
        items += [(name, tensor) for name, tensor in model.named_buffers() if name in persistent]
    elif isinstance(model, Mapping):
        items = list(_tensor_items(model))
    else:
        raise TypeError("Expected a tensor mapping or torch.nn.Module.")
    tensors = [(str(name), t) for name, t in items if torch.is_tensor(t) and t.is_floating_point()]
    if not tensors:
        raise ValueError("No floating tensors were found.")
    if len({name for name, _ in tensors}) != len(tensors):
        raise ValueError("Tensor names must be unique.")
    return tensors


def _floating_tensors(named_tensors):
    """Non-empty floating tensors, ordered by name (setup's visiting order)."""
    return [(name, t) for name, t in sorted(named_tensors, key=lambda item: item[0])
            if torch.is_tensor(t) and t.is_floating_point() and t.numel()]


def _stream_chunk_size(chunk_size, element_size):
    """Elements per source chunk: a chunk is `chunk_size` bytes of elements."""
    return max(1, chunk_size // int(element_size))


def time_call(func, /, *args, **kwargs):
    """(func(*args, **kwargs), elapsed seconds)."""
    start = time.perf_counter()
    result = func(*args, **kwargs)
    return result, time.perf_counter() - start
