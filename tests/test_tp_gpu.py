"""Tensor-parallel generation with compressed shards on two GPUs (NCCL).

Each rank slices a tiny Llama, compresses and decodes only its slices just
in time (overlapped schedule), and all-reduces after o_proj and down_proj.
Its logits and greedy tokens must equal the uncompressed tensor-parallel
model's bit for bit, and the ranks must agree. Skipped on boxes with fewer
than two GPUs."""

import copy
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, failures):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    try:
        from transformers import LlamaConfig, LlamaForCausalLM

        from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_model_for_gpu
        from neuralzip_b200.gpu.tp import assert_same_on_all_ranks, shard_for_tensor_parallel
        from neuralzip_b200.setup import NeuralZipSetup

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        config = LlamaConfig(vocab_size=256, hidden_size=512, intermediate_size=1408, num_hidden_layers=3,
                             num_attention_heads=8, num_key_value_heads=4)
        config._attn_implementation = "eager"
        torch.manual_seed(0)
        with torch.device("cuda", rank):
            model = LlamaForCausalLM(config).bfloat16().eval()
        shard_for_tensor_parallel(model, rank, world)
        uncompressed = copy.deepcopy(model)
        prompt = torch.arange(16, device=f"cuda:{rank}").reshape(1, -1) % 256
        with torch.no_grad():
            expected = uncompressed(prompt, use_cache=False).logits
            want = uncompressed.generate(prompt, max_new_tokens=8, min_new_tokens=8, do_sample=False,
                                         pad_token_id=0)
        setup = NeuralZipSetup(chunk_size=64 << 10).build(model)
        runtime = NeuralZipRuntime.attach(model, export_model_for_gpu(model, setup), device=f"cuda:{rank}")
        for workspace in runtime.workspaces.values():
            workspace.view(torch.uint8).fill_(0xA5)
        with torch.no_grad():
            got = model(prompt, use_cache=False).logits
            tokens = model.generate(prompt, max_new_tokens=8, min_new_tokens=8, do_sample=False, pad_token_id=0)
        assert torch.equal(got.view(torch.int16), expected.view(torch.int16)), "logits differ"
        assert torch.equal(tokens, want), "tokens differ"
        assert_same_on_all_ranks(tokens)
        runtime.check_status()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # reported to the parent process
        failures.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.timeout(600)
def test_two_gpu_tensor_parallel_generation():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
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
