"""Hugging Face integration: compressed GPU inference and checkpoint format v3.

Behaviour of neuralzip/gpu/pretrained.py:1-479. ``enable(setup, device=)``
patches ``PreTrainedModel.save_pretrained`` / ``from_pretrained`` for the
process:

* an ordinary checkpoint loads through Transformers; its eligible weights
  are exported to the GPU tile layout and a NeuralZipRuntime is attached
  (``model.neuralzip_stats.representation == "gpu"``);
* ``save_pretrained`` writes storage format v2 as two uint8 safetensors
  tensors, ``__neuralzip__.storage.data`` (the blob) and
  ``__neuralzip__.storage.metadata`` (compact sorted JSON), next to the
  tensors left uncompressed, and sets ``config.neuralzip = {format:
  "neuralzip", version: 3, encoding: "storage", aliases, stats}`` for the
  write only (``representation == "storage"``);
* a checkpoint whose config carries that entry is decoded on the host
  cores (one native pass over its chunks), built by Transformers from the
  decoded state dict, and exported to the GPU again.

Structure: ``_Checkpoint`` knows the v3 layout (names, config entry,
reading the shards), ``_LoadOptions`` validates what ``from_pretrained``
may be given for a v3 checkpoint, and the stats of the GPU representation
are summed by ``_gpu_stats`` from the export's own byte counts. Saving a
model with a runtime materializes its weights with the next block decoding
on the GPU while the current one is copied out.
"""

from __future__ import annotations

import inspect
import json
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path

import torch

from neuralzip_b200.compressor import NeuralZipCompressor
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.gpu.inference import GPUEncodedSymbols, NeuralZipRuntime, export_model_for_gpu
from neuralzip_b200.payloads import NeuralZipStats
from neuralzip_b200.setup import NeuralZipSetup
from neuralzip_b200.utils import _model_tensors, time_call

STATS_ATTRIBUTE = "neuralzip_stats"
_MISSING = object()
_ORIGINAL = {}       # "save" / "load": the Transformers methods this module wraps
_HF_OPTIONS = {}     # setup and default device given to enable()


class _Checkpoint:
    """The v3 layout: two uint8 tensors and one config entry."""

    NAME = "neuralzip"
    VERSION = 3
    PREFIX = "__neuralzip__."
    DATA = PREFIX + "storage.data"
    METADATA = PREFIX + "storage.metadata"

    @classmethod
    def entry(cls, config):
        """The config's neuralzip entry, or None for an ordinary checkpoint."""
        entry = getattr(config, "neuralzip", None)
        if not isinstance(entry, dict) or entry.get("format") != cls.NAME:
            return None
        version = entry.get("version")
        if type(version) is not int or version != cls.VERSION:
            raise ValueError("Unsupported NeuralZip checkpoint.")
        if entry.get("encoding") != "storage":
            raise ValueError("Invalid NeuralZip checkpoint format metadata.")
        return entry

    @classmethod
    def make_entry(cls, aliases, stats):
        return {"format": cls.NAME, "version": cls.VERSION, "encoding": "storage", "aliases": aliases,
                "stats": asdict(stats)}

    @classmethod
    def metadata_tensor(cls, metadata):
        text = json.dumps(metadata, separators=(",", ":"), sort_keys=True).encode("utf-8")
        return torch.frombuffer(bytearray(text), dtype=torch.uint8)

    @classmethod
    def read(cls, directory):
        """(blob tensor, storage metadata, resident tensors) of a v3 directory."""
        from safetensors.torch import load_file
        from transformers.utils import SAFE_WEIGHTS_INDEX_NAME, SAFE_WEIGHTS_NAME

        index = directory / SAFE_WEIGHTS_INDEX_NAME
        if index.is_file():
            weight_map = json.loads(index.read_text(encoding="utf-8"))["weight_map"]
            files = [directory / name for name in dict.fromkeys(weight_map.values())]
        else:
            files = [directory / SAFE_WEIGHTS_NAME]
        tensors = {}
        for path in files:
            shard = load_file(path, device="cpu")
            if tensors.keys() & shard.keys():
                raise ValueError("A checkpoint tensor occurs in more than one shard.")
            tensors.update(shard)
        special = {name for name in tensors if name.startswith(cls.PREFIX)}
        if special != {cls.DATA, cls.METADATA}:
            raise ValueError("The NeuralZip storage checkpoint is incomplete.")
        metadata = json.loads(tensors.pop(cls.METADATA).contiguous().numpy().tobytes().decode("utf-8"))
        return tensors.pop(cls.DATA), metadata, tensors


def _setup_seconds(setup):
    return 0.0 if setup is None else float(NeuralZipSetup.load(setup).setup_seconds or 0.0)


def _aliases(model):
    """Tied state entries: alias name -> the first name of the same tensor."""
    state = set(model.state_dict())
    aliases = {}
    for named in (model.named_parameters(remove_duplicate=False), model.named_buffers(remove_duplicate=False)):
        first = {}
        for name, tensor in named:
            if name in state and first.setdefault(id(tensor), name) != name:
                aliases[name] = first[id(tensor)]
    return aliases


def _storage_key(tensor):
    """Identity of a tensor's bytes: views of the same bytes count once."""
    return tensor.device, tensor.data_ptr(), tuple(tensor.shape), tuple(tensor.stride()), tensor.dtype


def _distinct_bytes(tensors):
    seen = {}
    for tensor in tensors:
        seen.setdefault(_storage_key(tensor), tensor.numel() * tensor.element_size())
    return sum(seen.values())


@dataclass
class _GpuBytes:
    """Byte counts of the GPU representation: compressed groups, their
    decode tables and the tensors left resident."""

    raw: int = 0
    compressed: int = 0
    exponent_raw: int = 0
    exponent_compressed: int = 0
    exponent_defined: bool = True
    stream_raw: int = 0
    stream_compressed: int = 0
    exponent_tables: set = field(default_factory=set)

    def add_resident(self, tensor):
        size = tensor.numel() * tensor.element_size()
        self.raw += size
        self.compressed += size
        if tensor.is_floating_point() and tensor.numel():
            spec = DTYPES.get(tensor.dtype)
            if spec is None or spec.exponent_stream is None:
                self.exponent_defined = False
            else:
                self.exponent_raw += tensor.numel()
                self.exponent_compressed += tensor.numel()

    def add_group(self, group):
        encoded = group.encoded
        self.raw += encoded.raw_bytes
        self.compressed += encoded.compressed_bytes
        exponent_lane = encoded.dtype.exponent_stream
        for lane, stream in enumerate(encoded.streams):
            if isinstance(stream, GPUEncodedSymbols):
                self.stream_raw += stream.symbol_count
                self.stream_compressed += stream.compressed_bytes
                if lane == exponent_lane:
                    self.exponent_tables.add(group.codebook_id)
        if exponent_lane is None:
            self.exponent_defined = False
        else:
            stream = encoded.streams[exponent_lane]
            self.exponent_raw += encoded.numel
            self.exponent_compressed += stream.compressed_bytes if isinstance(stream, GPUEncodedSymbols) \
                else len(stream)


def _gpu_stats(model, exported, setup, encoding_seconds):
    """Stats of the GPU representation (neuralzip/gpu/pretrained.py:122-193).
    Compressed bytes count the uploaded tile layout (bitstream words with
    their padding, sub-stream lengths, tile offsets) and each decode table
    as the kernel stages it, so the values differ from the reference's
    layout (segment gaps, block positions) while meaning the same thing."""
    counts = _GpuBytes()
    compressed_names = {binding.tensor_name for binding in exported.bindings}
    seen = set()
    for name, tensor in model.state_dict().items():
        key = _storage_key(tensor)
        if name not in compressed_names and key not in seen:
            seen.add(key)
            counts.add_resident(tensor)
    for group in exported.groups:
        counts.add_group(group)
    tables = {group.codebook_id: 4 * group.codebook.table_words for group in exported.groups}
    return NeuralZipStats(
        setup_seconds=_setup_seconds(setup), encoding_seconds=float(encoding_seconds),
        raw_bytes=counts.raw, compressed_bytes=counts.compressed + sum(tables.values()),
        exponent_raw_bytes=counts.exponent_raw if counts.exponent_defined else None,
        exponent_compressed_bytes=counts.exponent_compressed + sum(tables[i] for i in counts.exponent_tables)
        if counts.exponent_defined else None,
        stream_raw_bytes=counts.stream_raw, stream_compressed_bytes=counts.stream_compressed + sum(tables.values()),
        representation="gpu")


def _export_stats(model, exported, setup, encoding_seconds):
    return _gpu_stats(model, exported, setup, encoding_seconds)


def _attach(model, setup, device):
    """Exports `model` for the GPU, records its stats and attaches a runtime."""
    exported, seconds = time_call(export_model_for_gpu, model, setup)
    setattr(model, STATS_ATTRIBUTE, _gpu_stats(model, exported, setup, seconds))
    if exported.groups:
        NeuralZipRuntime.attach(model, exported, device=device)
    elif device is not None:
        model.to(device).eval()
    return exported


# ---- save ----------------------------------------------------------------------

def _storage_of(model, setup):
    """(blob, storage metadata, resident state, aliases, byte sizes, seconds):
    every floating tensor of the model goes to storage (a runtime's weights
    materialized from the GPU first); everything else stays resident."""
    tensors = dict(_model_tensors(model))
    runtime = getattr(model, "neuralzip_runtime", None)
    if isinstance(runtime, NeuralZipRuntime):
        tensors.update(runtime.materialized_weights())
    named = tuple(sorted(tensors.items()))
    blob, metadata, sizes, seconds = NeuralZipCompressor(setup).encode(named)
    aliases = _aliases(model)
    stored = {name for name, _ in named}
    resident = {name: tensor for name, tensor in model.state_dict().items()
                if name not in aliases and name not in stored and aliases.get(name, name) not in stored}
    extra = _distinct_bytes(resident.values())
    sizes["raw_bytes"] += extra
    sizes["compressed_bytes"] += extra
    return blob, metadata, resident, aliases, sizes, seconds


def _save_options(model, directory, save_args, save_kwargs):
    """The keyword arguments Transformers' save_pretrained receives, with the
    options NeuralZip cannot honour rejected."""
    bound = inspect.signature(_ORIGINAL["save"]).bind(model, directory, *save_args, **dict(save_kwargs or {}))
    bound.apply_defaults()
    options = dict(bound.arguments.pop("kwargs"))
    options.update(bound.arguments)
    for name in ("self", "save_directory"):
        options.pop(name)
    if options.pop("state_dict") is not None:
        raise ValueError("NeuralZip cannot compress an alternate state_dict.")
    if options.pop("variant", None) is not None:
        raise ValueError("NeuralZip checkpoints do not support variant filenames.")
    if options.pop("distributed_checkpoint", False):
        raise ValueError("NeuralZip does not support distributed checkpoint saving.")
    options["save_original_format"] = False
    return options


def _save_pretrained(model, directory, *, setup=None, save_args=(), save_kwargs=None):
    blob, metadata, resident, aliases, sizes, seconds = _storage_of(model, setup)
    stats = NeuralZipStats(setup_seconds=_setup_seconds(setup), encoding_seconds=float(seconds), **sizes)
    setattr(model, STATS_ATTRIBUTE, stats)
    options = _save_options(model, directory, save_args, save_kwargs)
    state = {**resident, _Checkpoint.DATA: blob, _Checkpoint.METADATA: _Checkpoint.metadata_tensor(metadata)}
    config = model.config
    previous = getattr(config, "neuralzip", _MISSING)
    config.neuralzip = _Checkpoint.make_entry(aliases, stats)
    try:
        return _ORIGINAL["save"](model, directory, state_dict=state, **options)
    finally:
        if previous is _MISSING:
            delattr(config, "neuralzip")
        else:
            config.neuralzip = previous


# ---- load ----------------------------------------------------------------------

_HUB_KEYS = ("revision", "token", "cache_dir", "local_files_only", "force_download")


def _device_of(value):
    """A CUDA device from from_pretrained's device_map (None/"auto": enable()'s)."""
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


@dataclass
class _LoadOptions:
    """What from_pretrained may be given for a v3 checkpoint."""

    device: object
    hub: dict
    subfolder: str
    dtype: object
    attn_implementation: object
    output_loading_info: bool

    @classmethod
    def parse(cls, kwargs):
        kwargs = dict(kwargs)
        device = _device_of(kwargs.pop("device_map", None))
        hub = {name: kwargs.pop(name) for name in _HUB_KEYS if name in kwargs}
        subfolder = kwargs.pop("subfolder", "")
        if kwargs.pop("use_safetensors", True) is False:
            raise ValueError("NeuralZip checkpoints require Safetensors.")
        dtype, torch_dtype = kwargs.pop("dtype", None), kwargs.pop("torch_dtype", None)
        if kwargs.pop("ignore_mismatched_sizes", False):
            raise ValueError("NeuralZip cannot ignore mismatched tensor sizes.")
        adapter = kwargs.pop("adapter_kwargs", None)
        if adapter and "_adapter_model_path" in adapter:
            raise ValueError("NeuralZip checkpoints do not support PEFT adapters.")
        output_loading_info = kwargs.pop("output_loading_info", False)
        attn_implementation = kwargs.pop("attn_implementation", None)
        for ignored in ("weights_only", "trust_remote_code", "_from_auto"):
            kwargs.pop(ignored, None)
        if kwargs:
            raise TypeError(f"Unsupported NeuralZip loading options: {', '.join(sorted(kwargs))}.")
        return cls(device, hub, subfolder, torch_dtype if dtype is None else dtype, attn_implementation,
                   output_loading_info)


def _directory(source, subfolder, hub):
    path = Path(source).expanduser()
    if not path.is_dir():
        from huggingface_hub import snapshot_download

        pattern = f"{subfolder}/*" if subfolder else "*"
        path = Path(snapshot_download(repo_id=str(source), allow_patterns=(f"{pattern}.json", f"{pattern}.safetensors"),
                                      **hub))
    return path / subfolder


def _decoded_state(blob, metadata, resident, aliases):
    state = dict(resident)
    state.update(NeuralZipCompressor().decode(blob, metadata))
    for alias, canonical in aliases.items():
        state[alias] = state[canonical]
    return state


def _load_storage(directory, device, model_class, model_args, config, entry, setup, dtype,
                  attn_implementation=None):
    from transformers import GenerationConfig

    blob, metadata, resident = _Checkpoint.read(directory)
    aliases = entry.get("aliases", {})
    state, decoding_seconds = time_call(_decoded_state, blob, metadata, resident, aliases)
    model, info = _ORIGINAL["load"](model_class, None, *model_args, config=config, state_dict=state, dtype=dtype,
                                     attn_implementation=attn_implementation, output_loading_info=True)
    if any(info.values()):
        raise ValueError("The decoded state does not match the model architecture.")
    if dtype in (None, "auto"):
        # Transformers picks one dtype; storage keeps each tensor's own dtype and bits.
        model.load_state_dict(state, assign=True)
        for alias, canonical in aliases.items():
            owner, _, attr = alias.rpartition(".")
            source, _, source_attr = canonical.rpartition(".")
            setattr(model.get_submodule(owner), attr, getattr(model.get_submodule(source), source_attr))
    model.config.name_or_path = str(directory)
    if (directory / "generation_config.json").is_file():
        model.generation_config = GenerationConfig.from_pretrained(directory, local_files_only=True)
    exported, runtime_encoding_seconds = time_call(export_model_for_gpu, model, setup)
    if exported.groups:
        NeuralZipRuntime.attach(model, exported, device=device)
    elif device is not None:
        model.to(device).eval()
    setattr(model, STATS_ATTRIBUTE, replace(NeuralZipStats(**entry["stats"]), decoding_seconds=decoding_seconds,
                                            runtime_encoding_seconds=runtime_encoding_seconds))
    return model


def _v3_config(cls, source, config, kwargs):
    """The config to load with when the checkpoint is v3, else None."""
    from transformers import AutoConfig

    if _Checkpoint.entry(config) is not None:
        return config
    hub = {name: kwargs[name] for name in _HUB_KEYS if name in kwargs}
    try:
        found = (getattr(cls, "config_class", None) or AutoConfig).from_pretrained(
            source, subfolder=kwargs.get("subfolder", ""), **hub)
    except (OSError, ValueError):
        return None
    return found if _Checkpoint.entry(found) is not None else None


def _patched_save(model, directory, *args, **kwargs):
    return _save_pretrained(model, directory, setup=_HF_OPTIONS["setup"], save_args=args, save_kwargs=kwargs)


def _patched_load(cls, source, *model_args, config=None, **kwargs):
    v3 = _v3_config(cls, source, config, kwargs)
    if v3 is None:
        if kwargs.get("quantization_config") is not None or getattr(config, "quantization_config", None) is not None:
            raise ValueError("NeuralZip cannot attach to a quantized model.")
        device = _device_of(kwargs.pop("device_map", None))
        result = _ORIGINAL["load"](cls, source, *model_args, config=config, **kwargs)
        _attach(result[0] if isinstance(result, tuple) else result, _HF_OPTIONS["setup"], device)
        return result
    options = _LoadOptions.parse(kwargs)
    model = _load_storage(_directory(source, options.subfolder, options.hub), options.device, cls, model_args, v3,
                          _Checkpoint.entry(v3), _HF_OPTIONS["setup"], options.dtype,
                          attn_implementation=options.attn_implementation)
    if options.output_loading_info:
        return model, {"missing_keys": set(), "unexpected_keys": set(), "mismatched_keys": set(), "error_msgs": []}
    return model


def enable(setup=None, *, device=None):
    """Installs the integration for the current process (idempotent)."""
    from transformers import PreTrainedModel

    _HF_OPTIONS.update(setup=setup, device=device)
    if PreTrainedModel.save_pretrained is _patched_save:
        return
    if not _ORIGINAL:
        _ORIGINAL["save"] = PreTrainedModel.save_pretrained
        _ORIGINAL["load"] = PreTrainedModel.__dict__["from_pretrained"].__func__
    PreTrainedModel.save_pretrained = _patched_save
    PreTrainedModel.from_pretrained = classmethod(_patched_load)


# Names of the v3 layout, as module constants for callers.
FORMAT_NAME = _Checkpoint.NAME
FORMAT_VERSION = _Checkpoint.VERSION
PREFIX = _Checkpoint.PREFIX
STORAGE_DATA = _Checkpoint.DATA
STORAGE_METADATA = _Checkpoint.METADATA
