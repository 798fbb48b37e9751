"""Transparent Hugging Face integration (checkpoint format v3).

Same behaviour as neuralzip/gpu/pretrained.py:1-479. ``enable(setup,
device=)`` patches ``PreTrainedModel.save_pretrained`` / ``from_pretrained``
for the process:

* an ordinary checkpoint loads through Transformers, then its eligible
  weights are encoded to the GPU layout and attached to a NeuralZipRuntime
  (``model.neuralzip_stats.representation == "gpu"``);
* ``save_pretrained`` decodes the runtime's weights, runs the storage codec
  and writes the blob and JSON metadata as the uint8 safetensors tensors
  ``__neuralzip__.storage.data`` / ``__neuralzip__.storage.metadata``, with
  ``config.neuralzip = {format: "neuralzip", version: 3, encoding:
  "storage", aliases, stats}`` (representation "storage");
* a v3 checkpoint is recognised from its config, decoded on the CPU, built
  through Transformers with ``state_dict=`` and re-encoded for the GPU.
"""

from __future__ import annotations

import inspect
import json
from dataclasses import asdict, replace
from pathlib import Path

import torch

from neuralzip_b200.compressor import NeuralZipCompressor
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu.inference import GPUEncodedSymbols, NeuralZipRuntime, export_model_for_gpu
from neuralzip_b200.payloads import NeuralZipStats
from neuralzip_b200.setup import NeuralZipSetup
from neuralzip_b200.utils import _model_tensors, time_call

FORMAT_NAME = "neuralzip"
FORMAT_VERSION = 3
PREFIX = "__neuralzip__."
STORAGE_DATA = f"{PREFIX}storage.data"
STORAGE_METADATA = f"{PREFIX}storage.metadata"
STATS_ATTRIBUTE = "neuralzip_stats"
_MISSING = object()
_ORIGINAL_SAVE = None
_ORIGINAL_LOAD = None
_HF_OPTIONS = {}


def _tensor_bytes(tensor):
    return tensor.detach().cpu().contiguous().numpy().tobytes()


def _setup_seconds(setup):
    return 0.0 if setup is None else float(NeuralZipSetup.load(setup).setup_seconds or 0.0)


def _aliases(model):
    """Tied state entries: alias name -> canonical name."""
    state_names = set(model.state_dict())
    aliases = {}
    for values in (model.named_parameters(remove_duplicate=False), model.named_buffers(remove_duplicate=False)):
        canonical = {}
        for name, tensor in values:
            if name not in state_names:
                continue
            source = canonical.setdefault(id(tensor), str(name))
            if source != name:
                aliases[str(name)] = source
    return aliases


def _storage_key(tensor):
    return tensor.device, tensor.data_ptr(), tuple(tensor.shape), tuple(tensor.stride()), tensor.dtype


def _resident_bytes(tensors):
    seen, total = set(), 0
    for tensor in tensors:
        key = _storage_key(tensor)
        if key not in seen:
            seen.add(key)
            total += tensor.numel() * tensor.element_size()
    return total


def _encode_model_storage(model, setup, runtime=None):
    """Encodes all floating model state; keeps only auxiliary tensors resident."""
    named_tensors = dict(_model_tensors(model))
    if runtime is not None:
        named_tensors.update(runtime.materialized_weights())
    named_tensors = tuple(sorted(named_tensors.items()))
    blob, metadata, sizes, seconds = NeuralZipCompressor(setup).encode(named_tensors)
    encoded_names = {name for name, _ in named_tensors}
    aliases = _aliases(model)
    resident = {
        name: tensor for name, tensor in model.state_dict().items()
        if name not in aliases and name not in encoded_names and aliases.get(name, name) not in encoded_names
    }
    auxiliary = _resident_bytes(resident.values())
    sizes["raw_bytes"] += auxiliary
    sizes["compressed_bytes"] += auxiliary
    return blob, metadata, resident, aliases, sizes, seconds


def _decode_model_storage(blob, metadata, resident, aliases):
    state = dict(resident)
    state.update(NeuralZipCompressor().decode(blob, metadata))
    for alias, canonical in aliases.items():
        state[alias] = state[canonical]
    return state


def _checkpoint_metadata(config):
    metadata = getattr(config, "neuralzip", None)
    if not isinstance(metadata, dict) or metadata.get("format") != FORMAT_NAME:
        return None
    version = metadata.get("version")
    if type(version) is not int or version != FORMAT_VERSION:
        raise ValueError("Unsupported NeuralZip checkpoint.")
    if metadata.get("encoding") != "storage":
        raise ValueError("Invalid NeuralZip checkpoint format metadata.")
    return metadata


def _export_stats(model, exported, setup, encoding_seconds):
    """Stats of the GPU representation (neuralzip/gpu/pretrained.py:122-193).

    ``stream_compressed_bytes`` and ``compressed_bytes`` count the bytes of
    the uploaded tile layout (bitstream words with padding, sub-stream
    lengths, tile offsets) and the decode tables as staged by the kernel,
    so they differ from the reference's layout (segment gaps and block
    positions) while meaning the same thing: bytes of the uploaded GPU
    representation."""
    compressed_names = {binding.tensor_name for binding in exported.bindings}
    resident_bytes = resident_exponent_bytes = 0
    exponent_available = True
    seen = set()
    for name, tensor in model.state_dict().items():
        key = _storage_key(tensor)
        if name in compressed_names or key in seen:
            continue
        seen.add(key)
        resident_bytes += tensor.numel() * tensor.element_size()
        if tensor.is_floating_point() and tensor.numel():
            config = DTYPES.get(tensor.dtype)
            if config is None or config.exponent_stream is None:
                exponent_available = False
            else:
                resident_exponent_bytes += tensor.numel()
    exponent_raw_bytes = exponent_compressed_bytes = resident_exponent_bytes
    exponent_codebooks = set()
    stream_raw_bytes = stream_compressed_bytes = 0
    for group in exported.groups:
        encoded = group.encoded
        for stream_id, stream in enumerate(encoded.streams):
            if isinstance(stream, GPUEncodedSymbols):
                stream_raw_bytes += stream.symbol_count
                stream_compressed_bytes += stream.compressed_bytes
                if stream_id == encoded.dtype.exponent_stream:
                    exponent_codebooks.add(group.codebook_id)
        if encoded.dtype.exponent_stream is None:
            exponent_available = False
        else:
            stream = encoded.streams[encoded.dtype.exponent_stream]
            exponent_raw_bytes += encoded.numel
            exponent_compressed_bytes += (stream.compressed_bytes if isinstance(stream, GPUEncodedSymbols)
                                          else len(stream))
    codebooks = {group.codebook_id: group.codebook for group in exported.groups}
    table_sizes = {key: 4 * book.table_words for key, book in codebooks.items()}
    codebook_bytes = sum(table_sizes.values())
    stream_compressed_bytes += codebook_bytes
    exponent_compressed_bytes += sum(table_sizes[i] for i in exponent_codebooks)
    return NeuralZipStats(
        setup_seconds=_setup_seconds(setup),
        encoding_seconds=float(encoding_seconds),
        raw_bytes=resident_bytes + sum(group.encoded.raw_bytes for group in exported.groups),
        compressed_bytes=resident_bytes + sum(group.encoded.compressed_bytes for group in exported.groups)
        + codebook_bytes,
        exponent_raw_bytes=exponent_raw_bytes if exponent_available else None,
        exponent_compressed_bytes=exponent_compressed_bytes if exponent_available else None,
        stream_raw_bytes=stream_raw_bytes,
        stream_compressed_bytes=stream_compressed_bytes,
        representation="gpu",
    )


def _encode_export(model, setup):
    exported, encoding_seconds = time_call(export_model_for_gpu, model, setup)
    setattr(model, STATS_ATTRIBUTE, _export_stats(model, exported, setup, encoding_seconds))
    return exported


def _attach_export(model, exported, device):
    if exported.groups:
        NeuralZipRuntime.attach(model, exported, device=device)
    elif device is not None:
        model.to(device).eval()


def _checkpoint_directory(value, **hub_kwargs):
    path = Path(value).expanduser()
    if path.is_dir():
        return path
    from huggingface_hub import snapshot_download

    return Path(snapshot_download(repo_id=str(value), **hub_kwargs))


def _checkpoint_state(directory):
    from safetensors.torch import load_file
    from transformers.utils import SAFE_WEIGHTS_INDEX_NAME, SAFE_WEIGHTS_NAME

    special, resident = {}, {}
    index = directory / SAFE_WEIGHTS_INDEX_NAME
    if index.is_file():
        weight_map = json.loads(index.read_text(encoding="utf-8"))["weight_map"]
        files = tuple(directory / name for name in dict.fromkeys(weight_map.values()))
    else:
        files = (directory / SAFE_WEIGHTS_NAME,)
    for path in files:
        shard = load_file(path, device="cpu")
        if (set(special) | set(resident)) & set(shard):
            raise ValueError("A checkpoint tensor occurs in more than one shard.")
        for name, tensor in shard.items():
            (special if name.startswith(PREFIX) else resident)[name] = tensor
    return special, resident


def _save_pretrained(model, directory, *, setup=None, save_args=(), save_kwargs=None):
    runtime = getattr(model, "neuralzip_runtime", None)
    blob, storage, resident, aliases, sizes, seconds = _encode_model_storage(
        model, setup, runtime if isinstance(runtime, NeuralZipRuntime) else None)
    stats = NeuralZipStats(setup_seconds=_setup_seconds(setup), encoding_seconds=float(seconds), **sizes)
    setattr(model, STATS_ATTRIBUTE, stats)
    bound = inspect.signature(_ORIGINAL_SAVE).bind(model, directory, *save_args, **dict(save_kwargs or {}))
    bound.apply_defaults()
    options = dict(bound.arguments.pop("kwargs"))
    options.update(bound.arguments)
    options.pop("self")
    options.pop("save_directory")
    if options.pop("state_dict") is not None:
        raise ValueError("NeuralZip cannot compress an alternate state_dict.")
    if options.pop("variant", None) is not None:
        raise ValueError("NeuralZip checkpoints do not support variant filenames.")
    if options.pop("distributed_checkpoint", False):
        raise ValueError("NeuralZip does not support distributed checkpoint saving.")
    state = dict(resident)
    state[STORAGE_DATA] = blob
    state[STORAGE_METADATA] = torch.frombuffer(bytearray(json.dumps(storage, separators=(",", ":"), sort_keys=True).encode("utf-8")), dtype=torch.uint8)
    metadata = {"format": FORMAT_NAME, "version": FORMAT_VERSION, "encoding": "storage", "aliases": aliases,
                "stats": asdict(stats)}
    config = model.config
    previous = getattr(config, "neuralzip", _MISSING)
    config.neuralzip = metadata
    options["save_original_format"] = False
    try:
        return _ORIGINAL_SAVE(model, directory, state_dict=state, **options)
    finally:
        if previous is _MISSING:
            delattr(config, "neuralzip")
        else:
            config.neuralzip = previous


def _load_storage(directory, device, model_class, model_args, config, metadata, setup, dtype,
                  attn_implementation=None):
    from transformers import GenerationConfig

    special, resident = _checkpoint_state(directory)
    if set(special) != {STORAGE_DATA, STORAGE_METADATA}:
        raise ValueError("The NeuralZip storage checkpoint is incomplete.")
    storage = json.loads(_tensor_bytes(special[STORAGE_METADATA]).decode("utf-8"))
    state, decoding_seconds = time_call(_decode_model_storage, special[STORAGE_DATA], storage, resident,
                                        metadata.get("aliases", {}))
    model, loading_info = _ORIGINAL_LOAD(model_class, None, *model_args, config=config, state_dict=state, dtype=dtype,
                                         attn_implementation=attn_implementation, output_loading_info=True)
    if any(loading_info.values()):
        raise ValueError("The decoded state does not match the model architecture.")
    if dtype in (None, "auto"):
        # Transformers infers one dtype; storage preserves each tensor's dtype and bits.
        model.load_state_dict(state, assign=True)
        for alias, canonical in metadata.get("aliases", {}).items():
            parent, _, name = alias.rpartition(".")
            source_parent, _, source_name = canonical.rpartition(".")
            setattr(model.get_submodule(parent), name, getattr(model.get_submodule(source_parent), source_name))
    model.config.name_or_path = str(directory)
    if (directory / "generation_config.json").is_file():
        model.generation_config = GenerationConfig.from_pretrained(directory, local_files_only=True)
    exported, runtime_encoding_seconds = time_call(export_model_for_gpu, model, setup)
    _attach_export(model, exported, device)
    stats = replace(NeuralZipStats(**metadata["stats"]), decoding_seconds=decoding_seconds,
                    runtime_encoding_seconds=runtime_encoding_seconds)
    setattr(model, STATS_ATTRIBUTE, stats)
    return model


def _patched_save(model, directory, *args, **kwargs):
    return _save_pretrained(model, directory, setup=_HF_OPTIONS["setup"], save_args=args, save_kwargs=kwargs)


def _load_device(kwargs):
    value = kwargs.pop("device_map", None)
    if value in (None, "auto"):
        return _HF_OPTIONS["device"]
    if isinstance(value, int):
        return f"cuda:{value}"
    try:
        device = torch.device(value)
    except (RuntimeError, TypeError) as error:
        raise TypeError("NeuralZip inference needs one CUDA device.") from error
    if device.type != "cuda":
        raise TypeError("NeuralZip inference needs one CUDA device.")
    return device


def _patched_load(cls, source, *model_args, config=None, **kwargs):
    from transformers import AutoConfig

    hub_keys = ("revision", "token", "cache_dir", "local_files_only", "force_download")
    hub = {name: kwargs[name] for name in hub_keys if name in kwargs}
    if _checkpoint_metadata(config) is None:
        config_class = getattr(cls, "config_class", None) or AutoConfig
        try:
            source_config = config_class.from_pretrained(source, subfolder=kwargs.get("subfolder", ""), **hub)
        except (OSError, ValueError):
            source_config = None
        if _checkpoint_metadata(source_config) is not None:
            config = source_config
    if _checkpoint_metadata(config) is None:
        if kwargs.get("quantization_config") is not None or getattr(config, "quantization_config", None) is not None:
            raise ValueError("NeuralZip cannot attach to a quantized model.")
        device = _load_device(kwargs)
        result = _ORIGINAL_LOAD(cls, source, *model_args, config=config, **kwargs)
        model = result[0] if isinstance(result, tuple) else result
        _attach_export(model, _encode_export(model, _HF_OPTIONS["setup"]), device)
        return result
    device = _load_device(kwargs)
    output_loading_info = kwargs.pop("output_loading_info", False)
    if kwargs.pop("use_safetensors", True) is False:
        raise ValueError("NeuralZip checkpoints require Safetensors.")
    dtype = kwargs.pop("dtype", None)
    attn_implementation = kwargs.pop("attn_implementation", None)
    torch_dtype = kwargs.pop("torch_dtype", None)
    if dtype is None:
        dtype = torch_dtype
    if kwargs.pop("ignore_mismatched_sizes", False):
        raise ValueError("NeuralZip cannot ignore mismatched tensor sizes.")
    for key in ("weights_only", "trust_remote_code", "_from_auto"):
        kwargs.pop(key, None)
    adapter_kwargs = kwargs.pop("adapter_kwargs", None)
    if adapter_kwargs and "_adapter_model_path" in adapter_kwargs:
        raise ValueError("NeuralZip checkpoints do not support PEFT adapters.")
    unsupported = sorted(set(kwargs) - set(hub_keys) - {"subfolder"})
    if unsupported:
        raise TypeError(f"Unsupported NeuralZip loading options: {', '.join(unsupported)}.")
    subfolder = kwargs.get("subfolder", "")
    pattern = f"{subfolder}/*" if subfolder else "*"
    directory = _checkpoint_directory(source, allow_patterns=(f"{pattern}.json", f"{pattern}.safetensors"),
                                      **hub) / subfolder
    model = _load_storage(directory, device, cls, model_args, config, _checkpoint_metadata(config),
                          _HF_OPTIONS["setup"], dtype, attn_implementation=attn_implementation)
    if output_loading_info:
        return model, {"missing_keys": set(), "unexpected_keys": set(), "mismatched_keys": set(), "error_msgs": []}
    return model


def enable(setup=None, *, device=None):
    """Installs the integration for the current process (idempotent)."""
    from transformers import PreTrainedModel

    global _ORIGINAL_SAVE, _ORIGINAL_LOAD
    _HF_OPTIONS.update(setup=setup, device=device)
    if PreTrainedModel.save_pretrained is not _patched_save:
        if _ORIGINAL_SAVE is None:
            _ORIGINAL_SAVE = PreTrainedModel.save_pretrained
            _ORIGINAL_LOAD = PreTrainedModel.__dict__["from_pretrained"].__func__
        PreTrainedModel.save_pretrained = _patched_save
        PreTrainedModel.from_pretrained = classmethod(_patched_load)
