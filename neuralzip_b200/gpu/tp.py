"""Tensor-parallel generation with compressed weights, one process per GPU.

Each rank keeps only its slice of every decoder layer's linear weights, and
the runtime compresses and decodes only that slice just in time. The
exchange is one NCCL all-reduce after each row-parallel projection:

* column-parallel, sliced by output rows: q_proj/k_proj/v_proj, by whole
  heads (query heads and key/value heads both divide by the world size), and
  gate_proj/up_proj, by intermediate features;
* row-parallel, sliced by input columns: o_proj and down_proj, whose partial
  outputs are summed over the ranks by a forward hook.

Embeddings, norms and the LM head stay replicated, so every rank computes
the same logits and picks the same greedy tokens. Llama-family decoder
layers (self_attn.{q,k,v,o}_proj, mlp.{gate,up,down}_proj) are supported;
the attention reshapes heads with -1, so sliced projections need no change
to the module code.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

_COLUMN = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.gate_proj", "mlp.up_proj")
_ROW = ("self_attn.o_proj", "mlp.down_proj")


def _slice_linear(linear, rank, world, dim):
    """Keeps this rank's contiguous 1/world of `linear` along `dim`
    (0: output rows, 1: input columns)."""
    weight = linear.weight.detach()
    size = weight.shape[dim]
    if size % world:
        raise ValueError(f"{size} features do not divide over {world} ranks.")
    part = size // world
    piece = weight.narrow(dim, rank * part, part).contiguous()
    linear.weight = nn.Parameter(piece, requires_grad=False)
    if dim == 0:
        linear.out_features = part
        if linear.bias is not None:
            linear.bias = nn.Parameter(linear.bias.detach().narrow(0, rank * part, part).contiguous(),
                                       requires_grad=False)
    else:
        linear.in_features = part


def _all_reduce_hook(group):
    def hook(_module, _inputs, output):
        dist.all_reduce(output, group=group)
        return output

    return hook


def decoder_layers(model):
    """The model's decoder layers (model.model.layers for HF causal LMs)."""
    base = getattr(model, "model", model)
    layers = getattr(base, "layers", None)
    if layers is None:
        raise ValueError("No decoder layers found (expected model.model.layers).")
    return layers


def shard_for_tensor_parallel(model, rank, world, group=None):
    """Slices every decoder layer of `model` in place for `rank` of `world`
    and registers the all-reduce after each row-parallel projection.
    Returns the hook handles. The model's weights must be identical on every
    rank beforehand (same seed or same checkpoint)."""
    config = getattr(model, "config", None)
    if config is not None:
        for name in ("num_attention_heads", "num_key_value_heads", "intermediate_size"):
            value = getattr(config, name, None)
            if value is not None and value % world:
                raise ValueError(f"config.{name} = {value} does not divide over {world} ranks.")
    handles = []
    for layer in decoder_layers(model):
        for name in _COLUMN:
            _slice_linear(layer.get_submodule(name), rank, world, 0)
        for name in _ROW:
            module = layer.get_submodule(name)
            if module.bias is not None:
                raise ValueError("Row-parallel projections with a bias are not supported.")
            _slice_linear(module, rank, world, 1)
            if world > 1:
                handles.append(module.register_forward_hook(_all_reduce_hook(group)))
    return handles


def local_config(config, world):
    """The config of one rank's slice under `world`-way tensor parallelism:
    query heads, key/value heads and the MLP width divided by the world
    size, the head size kept (so o_proj reads heads x head_dim inputs)."""
    import copy

    for name in ("num_attention_heads", "num_key_value_heads", "intermediate_size"):
        if getattr(config, name) % world:
            raise ValueError(f"config.{name} = {getattr(config, name)} does not divide over {world} ranks.")
    local = copy.deepcopy(config)
    local.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
    local.num_attention_heads = config.num_attention_heads // world
    local.num_key_value_heads = config.num_key_value_heads // world
    local.intermediate_size = config.intermediate_size // world
    return local


def build_tensor_parallel(model_class, config, rank, world, *, dtype, device, seed=0, std=0.02, group=None):
    """This rank's slice of a `model_class(config)` built directly, without
    the full model: a model of the per-rank config (the shapes of a rank's
    q/k/v/gate/up rows and o/down columns) whose replicated parts
    (embeddings, norms, LM head) come from `seed` on every rank, and whose
    sliced projections are drawn N(0, std) from a seed of their own per
    (rank, layer, projection), with the all-reduce after each row-parallel
    projection. Returns (model, hook handles)."""
    torch.manual_seed(seed)
    with torch.device(device):
        model = model_class(local_config(config, world)).to(dtype).eval()
    handles = []
    with torch.no_grad():
        for index, layer in enumerate(decoder_layers(model)):
            for k, name in enumerate(_COLUMN + _ROW):
                linear = layer.get_submodule(name)
                g = torch.Generator(device=linear.weight.device).manual_seed(
                    (seed * 1_000_003 + rank) * 1_000_003 + index * 16 + k)
                linear.weight.copy_(torch.randn(linear.weight.shape, generator=g, device=linear.weight.device) * std)
            if world > 1:
                for name in _ROW:
                    handles.append(layer.get_submodule(name).register_forward_hook(_all_reduce_hook(group)))
    return model, handles


def assert_same_on_all_ranks(tensor, group=None):
    """Raises unless `tensor` is bit-identical on every rank (a cheap
    all-gather of its bytes)."""
    world = dist.get_world_size(group)
    flat = tensor.detach().contiguous().view(torch.uint8).reshape(-1)
    gathered = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(gathered, flat, group=group)
    if not all(torch.equal(flat, other) for other in gathered):
        raise AssertionError("Ranks disagree.")
