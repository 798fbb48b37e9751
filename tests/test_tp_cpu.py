"""Tensor-parallel sharding (neuralzip_b200.gpu.tp) as two gloo ranks on CPU.

The sharded model's logits equal the unsharded model's up to the order of
the fp32 sums (the all-reduce adds two partial products), every rank gets
the same logits bit for bit, and each rank's compressed export covers
exactly its weight slices and decodes (oracle tile reader) to them."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_llama(dtype):
    from transformers import LlamaConfig, LlamaForCausalLM

    config = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                         num_attention_heads=8, num_key_value_heads=2)
    config._attn_implementation = "eager"
    torch.manual_seed(0)
    return LlamaForCausalLM(config).to(dtype).eval()


def _worker(rank, world, port, failures):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        import helpers as H
        from neuralzip_b200.gpu.inference import export_model_for_gpu
        from neuralzip_b200.gpu.tp import assert_same_on_all_ranks, shard_for_tensor_parallel
        from neuralzip_b200.setup import NeuralZipSetup
        from oracle import oracle as O

        dist.init_process_group("gloo", rank=rank, world_size=world)
        tokens = torch.arange(12).reshape(1, -1)
        full = _tiny_llama(torch.float32)
        with torch.no_grad():
            expected = full(tokens, use_cache=False).logits
        model = _tiny_llama(torch.float32)
        shard_for_tensor_parallel(model, rank, world)
        layer = model.model.layers[0]
        assert layer.self_attn.q_proj.weight.shape == (128 // world, 128)
        assert layer.mlp.down_proj.weight.shape == (128, 256 // world)
        with torch.no_grad():
            got = model(tokens, use_cache=False).logits
        assert torch.allclose(got, expected, rtol=1e-4, atol=1e-5), (got - expected).abs().max()
        assert_same_on_all_ranks(got)
        # This rank's compressed export holds its slices and decodes to them.
        shard = _tiny_llama(torch.bfloat16)
        shard_for_tensor_parallel(shard, rank, world)
        params = dict(shard.named_parameters())
        setup = NeuralZipSetup(chunk_size=8192).build(shard)
        export = export_model_for_gpu(shard, setup)
        names = {b.tensor_name for b in export.bindings}
        assert {n for n in names if ".layers." in n} == {
            n for n in params if ".layers." in n and n.endswith("proj.weight")}
        for group in export.groups:
            binding = group.bindings[0]
            start = group.workspace_offset - binding.workspace_offset
            spec = group.encoded.dtype
            raw = params[binding.tensor_name].detach().reshape(-1)[start:start + group.encoded.numel]
            raw = raw.view(torch.uint8).numpy().tobytes()
            sym = group.encoded.symbols
            if group.codebook.max_bits:
                sel = O.tile_decode(np.frombuffer(sym.bitstream, dtype=np.uint32),
                                    np.frombuffer(sym.lane_bits, np.uint16), np.asarray(sym.tile_offsets),
                                    group.encoded.numel, group.codebook.code_lengths, group.codebook.code_values,
                                    group.codebook.vocab)
            else:
                sel = np.frombuffer(sym.bitstream, dtype=np.uint8)
            assert np.array_equal(sel, H.selected_lane(raw, spec))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # reported to the parent process
        failures.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.timeout(600)
def test_two_rank_tensor_parallel_sharding():
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(540)
    for p in procs:
        if p.is_alive():
            p.kill()
    messages = []
    while not failures.empty():
        messages.append(failures.get())
    assert not messages, messages
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def _build_worker(rank, world, port, failures):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        from transformers import LlamaConfig, LlamaForCausalLM

        from neuralzip_b200.gpu.tp import assert_same_on_all_ranks, build_tensor_parallel

        dist.init_process_group("gloo", rank=rank, world_size=world)
        config = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                             num_attention_heads=8, num_key_value_heads=2)
        config._attn_implementation = "eager"
        model, handles = build_tensor_parallel(LlamaForCausalLM, config, rank, world, dtype=torch.float32,
                                               device="cpu", seed=3)
        assert len(handles) == 2 * config.num_hidden_layers
        layer = model.model.layers[0]
        assert layer.self_attn.q_proj.weight.shape == (128 // world, 128)
        assert layer.self_attn.k_proj.weight.shape == (2 * 16 // world, 128)
        assert layer.self_attn.o_proj.weight.shape == (128, 128 // world)
        assert layer.mlp.down_proj.weight.shape == (128, 256 // world)
        for name in ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight",
                     "model.layers.1.input_layernorm.weight"):
            assert_same_on_all_ranks(model.get_parameter(name))
        tokens = torch.arange(12).reshape(1, -1)
        with torch.no_grad():
            got = model(tokens, use_cache=False).logits
        assert_same_on_all_ranks(got)
        # The slices of all ranks put together form an ordinary model with
        # the same logits (up to the order of the fp32 sums).
        full = LlamaForCausalLM(config).eval()
        state = dict(model.state_dict())
        with torch.no_grad():
            for name, tensor in list(state.items()):
                if not name.endswith("proj.weight"):
                    continue
                parts = [torch.empty_like(tensor) for _ in range(world)]
                dist.all_gather(parts, tensor.contiguous())
                row = any(name.endswith(f"{p}.weight") for p in ("o_proj", "down_proj"))
                state[name] = torch.cat(parts, dim=1 if row else 0)
            full.load_state_dict(state)
            want = full(tokens, use_cache=False).logits
        assert torch.allclose(got, want, rtol=1e-4, atol=1e-5), (got - want).abs().max()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        failures.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.timeout(600)
def test_two_rank_tensor_parallel_built_per_rank():
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_build_worker, args=(r, 2, port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(540)
    for p in procs:
        if p.is_alive():
            p.kill()
    messages = []
    while not failures.empty():
        messages.append(failures.get())
    assert not messages, messages
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
