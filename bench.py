"""Bulk decode benchmark: decoded weight GB/s of NeuralZip's decompression
hot path on B200 (BASELINE.json metric), one process per GPU.

Workload (the mixed-coding stress case): 64 bf16
tensors of 2048 x 8192 whose 256 KiB chunks each draw sigma from
{0.002, 0.02, 0.2, 1.0}, plus one fp16 and one fp32 4096 x 4096 tensor of
N(0, 0.02); default NeuralZipSetup (JS clustering, up to 254 pairs). Data
are synthetic (seeded); rank r uses seed 1 + r, so N ranks decode N disjoint
workloads with no collective (weak scaling).

A step decodes every chunk once: a bf16 launch, and one launch mixing the
fp16 and fp32 groups (each CTA names its element layout) enqueued at once on
a low-priority side stream, as nz_decode_launch_many runs them. `value`
is decoded bytes of all ranks / the slowest rank's step time, inputs
resident in HBM (2.2 GB of outputs and 1.4 GB of inputs per rank, larger
than L2, so no flush is needed). `e2e` times the same decode through the
public runtime with the compressed arena copied host->device from pinned
memory and every decoded weight copied back to pinned host memory each step.

`--impl reference` times the reference's own CPU decode path for the same
chunks (oracle/_ref: the reference's decode_mixed_block_into,
restore_mixed_stream_chunk and run_parallel_jobs compiled from its sources)
on the host cores; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decoded weight GB/s (bulk decode, config 2: mixed-coding stress)"
SIGMAS = (0.002, 0.02, 0.2, 1.0)
CHUNK_ELEMS_BF16 = 131072


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--bf16-tensors", type=int, default=64, help="config 2 has 64")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-pieces", type=int, default=16, help="pipeline pieces of the host-to-host decode")
    p.add_argument("--workload", choices=("config2", "config3", "config4"), default="config2",
                   help="config2: bulk decode (default line); config3/4: batch-1 generation")
    p.add_argument("--new-tokens", type=int, default=None)
    p.add_argument("--no-overlap", action="store_true", help="sequential decode schedule")
    p.add_argument("--prefetch-depth", type=int, default=2, help="decode buffers per dtype in the overlapped schedule")
    p.add_argument("--blocks-per-launch", type=int, default=0,
                   help="consecutive blocks decoded by one launch (0 = auto)")
    p.add_argument("--batch", type=int, default=1, help="generation batch (config 4 also names 8)")
    p.add_argument("--gen-reps", type=int, default=3, help="alternating timed runs per model")
    p.add_argument("--tp", action="store_true", help="generation workloads: tensor parallel over the torchrun ranks")
    return p.parse_args()


def config2(seed, bf16_tensors=64):
    """Config 2 tensors from one generator."""
    g = torch.Generator().manual_seed(seed)
    sigma_index = torch.randint(len(SIGMAS), (bf16_tensors * 128,), generator=g)
    sigmas = torch.tensor(SIGMAS)[sigma_index]
    named = {}
    for t in range(bf16_tensors):
        w = torch.randn(2048, 8192, generator=g)
        w.view(128, -1).mul_(sigmas[t * 128:(t + 1) * 128, None])
        named[f"layers.{t}.weight"] = w.to(torch.bfloat16)
    named["fp16.weight"] = (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.float16)
    named["fp32.weight"] = torch.randn(4096, 4096, generator=g) * 0.02
    return named


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"nz_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.index)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = [line.split(",") for line in self.path.read_text().splitlines() if line.strip()]
        self.path.unlink(missing_ok=True)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({name for r in rows if len(r) >= 9 for name, v in zip(names, r[5:9])
                          if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch.distributed as dist

    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def algorithmic_bytes(groups):
    """Bytes one launch must move: compressed stream + sync metadata + raw
    lanes + decoded output per group, and each decode table once."""
    total = 0
    tables = {}
    for group in groups:
        enc = group.encoded
        sym = enc.symbols
        es = enc.dtype.element_size
        if group.codebook.max_bits:
            total += (sym.bit_length + 7) // 8 + len(sym.lane_bits) + 4 * len(sym.tile_offsets)
            tables[group.codebook_id] = 4 * group.codebook.table_words
        else:
            total += enc.numel
        total += (es - 1) * enc.numel + es * enc.numel
    return total + sum(tables.values())


# ---- CPU baseline: the reference's own CPU decode of mixed chunks -------------------

def cpu_sample(named, setup, max_chunks):
    """Storage-format frames of up to `max_chunks` mixed-coded bf16 chunks,
    encoded with the reference's own frame encoder; returns ctypes jobs."""
    from oracle import oracle as O

    from neuralzip_b200.compressor import NeuralZipCompressor
    from neuralzip_b200.dtypes import DTYPES

    spec = DTYPES[torch.bfloat16]
    comp = NeuralZipCompressor(setup)
    books = {p.codebook_id: p for p in comp.export_codebooks()}
    comp.prepare_storage_transfer_target([(n, t) for n, t in named.items() if t.dtype == torch.bfloat16])
    chunks, keep, decodebooks = [], [], {}
    for name, tensor in named.items():
        if tensor.dtype != torch.bfloat16:
            continue
        modes = comp._transfer_chunk_modes[comp._transfer_plan_key(name, tensor, 1)]
        raw = tensor.reshape(-1).view(torch.uint8).numpy()
        for c, mode in enumerate(modes):
            if mode["kind"] != "mixed_huffman" or len(chunks) >= max_chunks:
                continue
            part = raw[c * 2 * CHUNK_ELEMS_BF16:(c + 1) * 2 * CHUNK_ELEMS_BF16]
            lanes = O.split(part, spec)
            payload = books[mode["codebook_id"]]
            lengths = bytes(payload.codebook[4:])
            frame = np.frombuffer(O.ref_mixed_encode_native(lanes[1], lengths, bytes(payload.vocab)), dtype=np.uint8)
            if mode["codebook_id"] not in decodebooks:
                decodebooks[mode["codebook_id"]] = O.RefDecodebook(lengths, bytes(payload.vocab))
            out = np.empty(len(part), dtype=np.uint8)
            job = O.RefChunk()
            job.payload, job.payload_size = frame.ctypes.data, len(frame)
            job.book = decodebooks[mode["codebook_id"]].handle
            job.lanes[0] = lanes[0].ctypes.data
            job.out, job.numel, job.elem_size, job.reorder, job.stream_id = out.ctypes.data, len(lanes[0]), 2, 1, 1
            chunks.append(job)
            keep.append((frame, lanes, out, part))
    return chunks, keep, decodebooks


def time_cpu_reference(chunks, keep, seconds_target=10.0, threads=0):
    from oracle import oracle as O

    O.ref_decode_chunks(chunks, threads)  # warm-up + correctness
    for _frame, _lanes, out, part in keep:
        if not np.array_equal(out, part):
            raise AssertionError("reference CPU decode differs from the original chunk")
    decoded = sum(len(part) for *_, part in keep)
    reps, elapsed = 0, 0.0
    start = time.perf_counter()
    while elapsed < seconds_target:
        O.ref_decode_chunks(chunks, threads)
        reps += 1
        elapsed = time.perf_counter() - start
    return decoded * reps / elapsed / 1e9, decoded, reps, elapsed


def reference_threads():
    return min(os.cpu_count() or 1, 16)  # the reference pool caps at 16 (common.h:146)


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU decode on the host cores."""
    if rank != 0:
        return
    from oracle import oracle as O

    from neuralzip_b200.setup import NeuralZipSetup

    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (reference sources absent)"}))
        return
    named = config2(1, args.bf16_tensors)
    bf16 = {n: t for n, t in named.items() if t.dtype == torch.bfloat16}
    setup = NeuralZipSetup().build(bf16)
    chunks, keep, _books = cpu_sample(bf16, setup, max_chunks=512)
    threads = reference_threads()
    O.ref_decode_chunks(chunks, threads)
    decoded = sum(len(p) for *_, p in keep)
    for _ in range(args.warmup):
        O.ref_decode_chunks(chunks, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.ref_decode_chunks(chunks, threads)
        times.append(time.perf_counter() - t0)
    mean = sum(times) / len(times)
    value = decoded / mean / 1e9
    sample = (f"{len(chunks)} mixed-coded bf16 chunks of config 2 (seed 1), {decoded / 1e6:.0f} MB decoded per step, "
              "storage-format frames from the reference encoder")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": "config2-bf16-mixed-sample", "chunks": len(chunks), "threads": threads},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))



# ---- configs 3 and 4: batch-1 greedy generation -------------------------------------

def _model_config(name):
    from transformers import LlamaConfig, Qwen2Config

    if name == "config3":  # Qwen2.5-0.5B architecture
        return Qwen2Config(hidden_size=896, num_hidden_layers=24, num_attention_heads=14, num_key_value_heads=2,
                           intermediate_size=4864, vocab_size=151936, tie_word_embeddings=True,
                           max_position_embeddings=4096), 32, 128
    return LlamaConfig(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                       intermediate_size=14336, vocab_size=128256, max_position_embeddings=4096), 128, 256


def run_generation(args, world, rank, local):
    """Random-init model of the config's architecture (N(0, 0.02), norms 1),
    compressed through neuralzip.setup + the GPU export, then greedy
    generation with KV cache and eager attention. An uncompressed copy of
    the same model is timed alternately with the compressed one (medians of
    `--gen-reps` runs each, so drift of the host or the GPU hits both
    alike); both must generate the same tokens, and the first-step logits
    must be equal bit for bit."""
    import copy

    from transformers import AutoModelForCausalLM

    from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_model_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    config, prompt_len, new_tokens = _model_config(args.workload)
    new_tokens = args.new_tokens or new_tokens
    config._attn_implementation = "eager"  # the reference's GPU protocol (eager attention)
    torch.manual_seed(0)
    with torch.device(device):
        model = AutoModelForCausalLM.from_config(config, dtype=torch.bfloat16).eval()
    prompt = torch.randint(config.vocab_size, (args.batch, prompt_len),
                           generator=torch.Generator().manual_seed(1)).to(device)

    def run(m, n):
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        with torch.no_grad():
            out = m.generate(prompt, max_new_tokens=n, min_new_tokens=n, do_sample=False, use_cache=True,
                             pad_token_id=0)
        torch.cuda.synchronize(device)
        return out, time.perf_counter() - t0

    def generate(m):
        """Tokens and seconds per generation step after the first (prefill
        and per-call setup excluded by timing a one-token call too)."""
        out, full = run(m, new_tokens)
        _, one = run(m, 1)
        return out, (full - one) / (new_tokens - 1)

    tp = args.tp and world > 1
    if tp:  # tensor parallel over the torchrun ranks: each keeps and compresses its slices
        from neuralzip_b200.gpu.tp import assert_same_on_all_ranks, shard_for_tensor_parallel

        shard_for_tensor_parallel(model, rank, world)
        torch.cuda.empty_cache()
    with torch.no_grad():
        ref_logits = model(prompt, use_cache=False).logits.float().cpu()
    uncompressed = copy.deepcopy(model)
    t0 = time.perf_counter()
    setup = NeuralZipSetup().build(model)
    exported = export_model_for_gpu(model, setup)
    prep_s = time.perf_counter() - t0
    per_launch = "auto" if args.blocks_per_launch == 0 else args.blocks_per_launch
    runtime = NeuralZipRuntime.attach(model, exported, device=device, overlap=not args.no_overlap,
                                      prefetch_depth=args.prefetch_depth, blocks_per_launch=per_launch)
    with torch.no_grad():
        logits = model(prompt, use_cache=False).logits.float().cpu()
    identical = bool(torch.equal(logits.view(torch.int32), ref_logits.view(torch.int32)))
    generate(uncompressed)  # warm-up
    generate(model)
    ref_times, comp_times = [], []
    for _ in range(args.gen_reps):
        ref_tokens, t = generate(uncompressed)
        ref_times.append(t)
        tokens, t = generate(model)
        comp_times.append(t)
    ref_s, comp_s = statistics.median(ref_times), statistics.median(comp_times)
    if tp:
        assert_same_on_all_ranks(tokens)
        ref_s, comp_s = max_over_ranks(ref_s, world), max_over_ranks(comp_s, world)
    # Per-step decode work: one decode of every unit, as the schedule launches it.
    decode_ms = []
    stream = torch.cuda.current_stream(device)
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for unit in range(len(runtime._units)):
            runtime._decode_unit(unit, stream)
        b.record(stream)
        torch.cuda.synchronize(device)
        decode_ms.append(a.elapsed_time(b))
    decoded = sum(g.encoded.numel * g.encoded.dtype.element_size for g in exported.groups)
    if rank == 0:
        print(json.dumps({
            "metric": f"batch-{args.batch} greedy generation tok/s, compressed weights decoded per layer per step",
            "value": round(args.batch / comp_s, 3), "unit": "tok/s", "n_gpus": world if tp else 1,
            "higher_is_better": True, "parallelism": f"tp{world}, NCCL all-reduce after o_proj and down_proj"
            if tp else "single GPU",
            "workload": args.workload, "uncompressed_tok_s": round(args.batch / ref_s, 3),
            "ratio_vs_uncompressed": round(ref_s / comp_s, 4),
            "ratio_runs": [round(r / c, 4) for r, c in zip(ref_times, comp_times)],
            "tokens_identical": bool(torch.equal(tokens, ref_tokens)),
            "first_step_logits_bitwise": identical, "overlap": runtime.overlap,
            "prefetch_depth": runtime.prefetch_depth, "blocks_per_launch": runtime.blocks_per_launch,
            "launch_units": len(runtime._units),
            "decode_per_step_ms": round(min(decode_ms), 3),
            "decode_gbs": round(decoded / (min(decode_ms) * 1e-3) / 1e9, 1),
            "compressed_weights": len({b.tensor_name for b in exported.bindings}), "prep_s": round(prep_s, 1),
            "config": {"workload": args.workload, "batch": args.batch, "prompt": prompt_len,
                       "new_tokens": new_tokens, "attn": "eager", "kv_cache": True,
                       "timing": "(t(new_tokens) - t(1)) / (new_tokens - 1): prefill excluded; "
                                 f"median of {args.gen_reps} runs alternating with the uncompressed model"},
        }))


def main():
    args = parse_args()
    world, rank, local = dist_setup()
    if args.workload != "config2" or args.impl == "reference":
        if args.workload != "config2":
            run_generation(args, world, rank, local)
        else:
            run_reference(args, world, rank)
        barrier(world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_tensors_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    # Ranks share the host: each builds its workload on its share of the cores.
    host_threads = max(1, (os.cpu_count() or 1) // world)
    if world > 1:
        torch.set_num_threads(host_threads)
    t0 = time.perf_counter()
    named = config2(1 + rank, args.bf16_tensors)
    setup = NeuralZipSetup().build(named)
    t_setup = time.perf_counter() - t0
    export = export_tensors_for_gpu(named, setup, threads=host_threads)
    t_export = time.perf_counter() - t0 - t_setup
    runtime = NeuralZipRuntime(None, export, device)
    block = export.block_order[0]
    batches = runtime._prepared_batches[block]
    decoder = runtime._decoder
    stream = torch.cuda.current_stream(device)

    # Correctness of this very workload before timing: every tensor bit-exact.
    runtime._decode_block(block)
    torch.cuda.synchronize(device)
    views = {}
    for item in runtime._groups_by_block[block]:
        for binding in item.group.bindings:
            views[binding.tensor_name] = (item.group.encoded.dtype.torch_dtype, binding)
    for name, (dtype, binding) in views.items():
        got = runtime.workspaces[dtype][binding.workspace_offset:binding.workspace_offset + binding.numel]
        if not torch.equal(got.view(torch.uint8).cpu(), named[name].reshape(-1).view(torch.uint8)):
            raise AssertionError(f"decode of {name} is not bit-exact")
    runtime.check_status()

    decoded_bytes = sum(g.encoded.numel * g.encoded.dtype.element_size for g in export.groups)
    main_batch = max(batches, key=lambda b: b.elements)
    main_groups = [g for g in export.groups if g.encoded.dtype.name == "bfloat16"]
    alg_bytes = algorithmic_bytes(main_groups)

    # One step = the block's launches as TileDecoder.decode_batches runs
    # them: the bf16 launch alone on `stream` (timed for the roofline), then
    # one launch that mixes the fp16 and fp32 groups.
    others = [b for b in batches if b is not main_batch]
    sides = [torch.cuda.Stream(device=device, priority=0) for _ in others]
    fork = torch.cuda.Event()
    joins = [torch.cuda.Event() for _ in others]

    def step(times=None):
        # As nz_decode_launch_many runs them: the bf16 launch first, the
        # others enqueued at once on low-priority streams (they take SMs as
        # bf16 CTAs finish).
        fork.record(stream)
        if times is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
        decoder.decode_batch(main_batch, stream)
        if times is not None:
            b.record(stream)
            times.append((a, b))
        for side, join, batch in zip(sides, joins, others):
            side.wait_event(fork)
            decoder.decode_batch(batch, side)
            join.record(side)
            stream.wait_event(join)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    kernel_events = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        torch.cuda.synchronize(device)
        barrier(world)
        start.record(stream)
        for _ in range(args.steps):
            step(kernel_events)
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    step_ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    kernel_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kernel_events) / len(kernel_events), world)
    clock = clocks.summary()
    # The bf16 launch alone (no other launch sharing its tail), after the
    # timed region: the kernel's own rate, for the roofline beside the
    # in-step one.
    alone = []
    for _ in range(max(3, min(args.steps, 50))):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        decoder.decode_batch(main_batch, stream)
        b.record(stream)
        alone.append((a, b))
    torch.cuda.synchronize(device)
    alone_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in alone) / len(alone), world)

    # e2e: pinned host compressed arena -> device -> decode -> pinned host
    # decoded weights, through the public bulk API (pipelined pieces).
    e2e = None
    if not args.no_e2e:
        from neuralzip_b200.gpu.bulk import HostDecoder

        host = HostDecoder(export, device, pieces=args.e2e_pieces)
        for _ in range(max(3, args.warmup // 2)):
            host.decode(stream)
        torch.cuda.synchronize(device)
        barrier(world)
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_steps = max(3, args.steps // 8)
        e_start.record(stream)
        for _ in range(e_steps):
            host.decode(stream)
        e_end.record(stream)
        torch.cuda.synchronize(device)
        e_ms = max_over_ranks(e_start.elapsed_time(e_end) / e_steps, world)
        host.check_status()
        decoded = host.tensors()
        for name, tensor in named.items():
            if not torch.equal(decoded[name].reshape(-1).view(torch.uint8), tensor.reshape(-1).view(torch.uint8)):
                raise AssertionError(f"e2e decode of {name} is not bit-exact")
        e2e = {"value": round(decoded_bytes * world / (e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": host.h2d_bytes, "d2h_bytes_per_step": host.d2h_bytes,
               "ms_per_step": round(e_ms, 3),
               "path": f"HostDecoder: pinned host arena -> H2D -> tile decode -> D2H of every decoded weight, "
                       f"{len(host.pieces)} pieces pipelined on three streams"}
        del host

    peak, peak_kind = peaks()
    achieved = alg_bytes / (kernel_ms * 1e-3) / 1e9
    traffic = None
    traffic_file = ROOT / "profiles" / "nz_tile_decode_bf16_traffic.txt"
    if traffic_file.is_file():
        fields = {k.strip(): v.strip() for k, v in (line.split("=", 1) for line in traffic_file.read_text().splitlines()
                                                    if line.startswith(("dram_bytes_per_launch", "elements_per_launch")))}
        if len(fields) == 2:  # ncu capture of the full launch, scaled if the workload size differs
            per_elem = float(fields["dram_bytes_per_launch"]) / float(fields["elements_per_launch"])
            traffic = int(per_elem * main_batch.elements)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:  # the CPU baseline is an N=1 figure
        from oracle import oracle as O

        if O.ref_available():
            bf16 = {n: t for n, t in named.items() if t.dtype == torch.bfloat16}
            chunks, keep, _books = cpu_sample(bf16, setup, max_chunks=256)
            threads = reference_threads()
            gbs, sample_bytes, reps, elapsed = time_cpu_reference(chunks, keep, 10.0, threads)
            cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                   "sample": f"{len(chunks)} mixed-coded bf16 chunks ({sample_bytes / 1e6:.0f} MB decoded) x {reps} "
                             f"in {elapsed:.1f} s, reference decode_mixed_block_into + restore_mixed_stream_chunk"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(decoded_bytes * world / (step_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(step_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {
                "workload": "config2", "bf16_tensors": args.bf16_tensors, "decoded_bytes_per_gpu": decoded_bytes,
                "groups": len(export.groups), "launches_per_step": len(batches),
                "codebooks": sorted({(b.mode, len(b.vocab) // 2) for b in setup.codebooks}),
                "l2": "inputs and outputs larger than L2 (no flush)", "setup_s": round(t_setup, 1),
                "export_s": round(t_export, 1), "parallelism": f"{world} independent ranks",
                "host_cores": os.cpu_count(),
            },
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": "nz_tile_decode (bf16 launch)",
                         "kernel_ms": round(kernel_ms, 4),
                         "algorithmic_bytes": int(alg_bytes),
                         "alone": {"kernel_ms": round(alone_ms, 4),
                                   "achieved": round(alg_bytes / (alone_ms * 1e-3) / 1e9, 1),
                                   "frac": round(alg_bytes / (alone_ms * 1e-3) / 1e9 / peak, 4),
                                   "note": "the same launch timed by itself after the timed region; in the "
                                           "step the fp16+fp32 launch shares its tail"}},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clock,
            "gpu_launches": args.steps * len(batches),
        }
        print(json.dumps(line))
    barrier(world)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
