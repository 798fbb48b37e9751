"""Bulk decode benchmark: decoded weight GB/s of NeuralZip's decompression
hot path on B200 (BASELINE.json metric), one process per GPU.

N = 1 (the default line). Workload: BASELINE.json configs[1], the
mixed-coding stress case: 64 bf16 tensors of 2048 x 8192 whose 256 KiB
chunks each draw sigma from {0.002, 0.02, 0.2, 1.0}, plus one fp16 and one
fp32 4096 x 4096 tensor of N(0, 0.02); default NeuralZipSetup (JS
clustering, up to 254 pairs). A step decodes every chunk once: a bf16
launch, and one launch mixing the fp16 and fp32 groups enqueued at once on a
low-priority side stream, as nz_decode_launch_many runs them. `value` is
decoded bytes / step time, inputs resident in HBM (2.2 GB of outputs and
1.4 GB of inputs, larger than L2, so no flush is needed). The line also
carries, measured in the same run on the same GPU:
  * per_dtype: each dtype's groups decoded by a launch of their own;
  * config1: configs[0], one 4096 x 4096 bf16 tensor with singleton
    (Huff0) codebooks: one decode per launch over 16 rotating copies (so L2
    never holds the 56 MB it moves), replayed from a CUDA graph, and all
    copies in one launch; beside it the CPU decode of the same storage
    chunks (this build's RFC 8878 restatement), cold and warm;
  * generation: configs[2], Qwen2.5-0.5B architecture, batch-1 greedy
    generation of 128 tokens with per-layer decode; tokens and first-step
    logits must equal the uncompressed model's (asserted); tok/s of both
    models and GPU-busy ms per token of both (union of kernel intervals);
  * config5a_1gpu: one GPU's share of the multi-GPU workload below.

N > 1 (torchrun). Workload: configs[4] (a), Llama-3-70B-architecture decoder
layers (q/k/v/o/gate/up/down, N(0, 0.02)); the checkpoint has N x
--layers-per-gpu layers, cut into N contiguous chunk ranges balanced by
decoded bytes (the rule of neuralzip_b200.gpu.shard.partition), and each rank
generates, compresses, uploads and decodes only its own range: weak scaling,
no collective on the data path. `value` = decoded bytes of all ranks / the
slowest rank's step time (CUDA events, max over ranks).

`e2e` times the same decode through the public host-to-host API
(HostDecoder): the compressed arena copied host->device from pinned memory
and every decoded weight copied back to pinned host memory each step.

`--impl reference` times the reference's own CPU decode path (oracle/_ref:
the reference's decode_mixed_block_into, restore_mixed_stream_chunk and
run_parallel_jobs compiled from its sources) on a sample of the same
workload's mixed-coded chunks, on the host cores; under torchrun only rank 0
runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decoded weight GB/s (bulk decode)"
SIGMAS = (0.002, 0.02, 0.2, 1.0)
CHUNK_ELEMS_BF16 = 131072
# Llama-3-70B decoder layer: (module, (out, in)).
LLAMA70B_LAYER = (("self_attn.q_proj", (8192, 8192)), ("self_attn.k_proj", (1024, 8192)),
                  ("self_attn.v_proj", (1024, 8192)), ("self_attn.o_proj", (8192, 8192)),
                  ("mlp.gate_proj", (28672, 8192)), ("mlp.up_proj", (28672, 8192)),
                  ("mlp.down_proj", (8192, 28672)))


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--bf16-tensors", type=int, default=64, help="config 2 has 64")
    p.add_argument("--layers-per-gpu", type=int, default=1, help="config 5a layers per rank")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-config1", action="store_true")
    p.add_argument("--no-generation", action="store_true")
    p.add_argument("--no-config5a", action="store_true", help="N=1: skip the one-GPU share of config 5a")
    p.add_argument("--e2e-pieces", type=int, default=16, help="pipeline pieces of the host-to-host decode")
    p.add_argument("--workload", choices=("bulk", "config1", "config3", "config4", "config5b"), default="bulk",
                   help="bulk: config 2 at N=1, config 5a under torchrun (default line); config1: the single-tensor "
                        "singleton record alone; config3/4: generation; config5b: tensor-parallel generation over "
                        "the torchrun ranks, each building its slices")
    p.add_argument("--layers", type=int, default=None, help="config5b: decoder layers (80 in configs[4])")
    p.add_argument("--new-tokens", type=int, default=None)
    p.add_argument("--no-overlap", action="store_true", help="sequential decode schedule")
    p.add_argument("--prefetch-depth", type=int, default=2, help="decode buffers per dtype in the overlapped schedule")
    p.add_argument("--blocks-per-launch", type=int, default=0,
                   help="consecutive blocks decoded by one launch (0 = auto)")
    p.add_argument("--batch", type=int, default=1, help="generation batch (config 4 also names 8)")
    p.add_argument("--gen-reps", type=int, default=3, help="alternating timed runs per model")
    p.add_argument("--tp", action="store_true", help="generation workloads: tensor parallel over the torchrun ranks")
    p.add_argument("--cuda-graphs", action="store_true",
                   help="config3/config4: also time both models with the one-token step captured in a CUDA graph")
    return p.parse_args()


# ---- workloads ----------------------------------------------------------------------

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


def config1():
    """Config 1: one 4096 x 4096 bf16 tensor."""
    g = torch.Generator().manual_seed(0)
    return {"w": (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.bfloat16)}


def config5a_tensors(layers):
    """(name, shape, seed) of every weight of `layers` 70B-architecture
    decoder layers, in checkpoint order; each tensor has its own seed, so
    any rank can generate any tensor alone."""
    out = []
    for layer in range(layers):
        for k, (module, shape) in enumerate(LLAMA70B_LAYER):
            out.append((f"model.layers.{layer}.{module}.weight", shape, 7000 + layer * len(LLAMA70B_LAYER) + k))
    return out


def config5a_share(layers, rank, world):
    """This rank's chunks of the config-5a checkpoint: the contiguous range
    of 256 KiB chunks whose bounds are the chunk edges nearest to equal
    splits of the decoded bytes (neuralzip_b200.gpu.shard.partition's rule,
    applied to the shapes, so no rank needs another rank's data). Returns
    [(name, shape, seed, first_chunk, chunks)]."""
    from neuralzip_b200.gpu.shard import partition

    class _Chunk:  # what partition() reads of a group: its decoded size
        def __init__(self, numel):
            self.encoded = type("E", (), {"numel": numel, "dtype": type("D", (), {"element_size": 2})})

    tensors = config5a_tensors(layers)
    chunks = [(i, c) for i, (_, shape, _) in enumerate(tensors)
              for c in range(-(-shape[0] * shape[1] // CHUNK_ELEMS_BF16))]
    sizes = [_Chunk(min(CHUNK_ELEMS_BF16, tensors[i][1][0] * tensors[i][1][1] - c * CHUNK_ELEMS_BF16))
             for i, c in chunks]
    start, end = partition(sizes, world)[rank]
    share = {}
    for i, c in chunks[start:end]:
        first, count = share.get(i, (c, 0))
        share[i] = (first, count + 1)
    return [(tensors[i][0], tensors[i][1], tensors[i][2], first, count) for i, (first, count) in share.items()]


def config5a_generate(share, device):
    """The rank's tensors (its chunk range of each), N(0, 0.02) bf16, drawn
    on the GPU from each tensor's own seed and returned on the host."""
    named = {}
    for name, shape, seed, first, count in share:
        g = torch.Generator(device=device).manual_seed(seed)
        w = (torch.randn(shape, generator=g, device=device) * 0.02).to(torch.bfloat16).reshape(-1)
        lo, hi = first * CHUNK_ELEMS_BF16, min(w.numel(), (first + count) * CHUNK_ELEMS_BF16)
        key = name if (lo, hi) == (0, w.numel()) else f"{name}[{lo}:{hi}]"
        named[key] = w[lo:hi].cpu()
        del w
    torch.cuda.empty_cache()
    return named


_T0 = time.perf_counter()


def log(what):
    """Progress on stderr (the result line alone goes to stdout)."""
    sys.stderr.write(f"[bench {time.perf_counter() - _T0:7.1f}s] {what}\n")
    sys.stderr.flush()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# ---- clocks: in-process NVML polling (read-only) ----------------------------------------

class NvmlClocks:
    """Polls the GPU's SM clock and clock-event reasons every `period_s`
    through NVML (read-only queries) on a background thread; `timed()`
    brackets the regions whose samples the summary covers."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index, period_s=0.005):
        self.period = period_s
        self.samples = []   # (t, sm_mhz, reasons mask)
        self.windows = []   # (t0, t1) of timed regions
        self._stop = threading.Event()
        self._thread = None
        self.error = None
        try:
            import pynvml

            self._nvml = pynvml
            self._handle = torch.cuda._get_pynvml_handler(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: the line says so
            self._handle = None
            self.max_mhz = None
            self.error = f"{type(exc).__name__}: {exc}"

    def _reasons(self):
        n = self._nvml
        fn = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(self._handle))

    def _poll(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append((time.perf_counter(), n.nvmlDeviceGetClockInfo(self._handle, n.NVML_CLOCK_SM),
                                     self._reasons()))
            except Exception as exc:
                self.error = f"{type(exc).__name__}: {exc}"
                return
            self._stop.wait(self.period)

    def __enter__(self):
        if self._handle is not None:
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(2)

    class _Window:
        def __init__(self, owner):
            self.owner = owner

        def __enter__(self):
            self.t0 = time.perf_counter()

        def __exit__(self, *exc):
            self.owner.windows.append((self.t0, time.perf_counter()))

    def timed(self):
        return self._Window(self)

    def summary(self):
        inside = [s for s in self.samples if any(a <= s[0] <= b for a, b in self.windows)]
        reasons = sorted({name for _, _, mask in inside for bit, name in self.REASONS.items() if mask & bit})
        out = {"sm_mhz": statistics.median(s[1] for s in inside) if inside else None,
               "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(inside),
               "sm_mhz_min": min((s[1] for s in inside), default=None),
               "source": "in-process NVML polled every 5 ms during the timed regions"}
        if self.error:
            out["error"] = self.error
        return out


# ---- distributed plumbing --------------------------------------------------------------

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


def gather_over_ranks(value, world):
    if world == 1:
        return [value]
    import torch.distributed as dist

    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


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


def time_launches(fn, stream, launches, reps=5):
    """Median per-launch ms of `launches` back-to-back calls of fn, over reps."""
    out = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(launches):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b) / launches)
    return statistics.median(out)


def copy_bound(host, stream, reps=3):
    """The host links' bound on a host-to-host decode: the same bytes
    copied with no decode, H2D alone (compressed arena), D2H alone (decoded
    workspaces) and both at once on the HostDecoder's two copy streams;
    median ms of `reps` each."""
    rt = host.runtime

    def h2d():
        with torch.cuda.stream(host.h2d):
            rt.arena.copy_(host.host_arena, non_blocking=True)

    def d2h():
        with torch.cuda.stream(host.d2h):
            for dtype, out in host.host_outputs.items():
                out.copy_(rt.workspaces[dtype], non_blocking=True)

    def timed(copies):
        out = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for s in (host.h2d, host.d2h):
                s.wait_event(a)
            for copy in copies:
                copy()
            for s in (host.h2d, host.d2h):
                stream.wait_stream(s)
            b.record(stream)
            torch.cuda.synchronize()
            out.append(a.elapsed_time(b))
        return statistics.median(out)

    h2d_ms, d2h_ms, both_ms = timed((h2d,)), timed((d2h,)), timed((h2d, d2h))
    return {"h2d_ms": round(h2d_ms, 3), "h2d_gbs": round(host.h2d_bytes / h2d_ms / 1e6, 2),
            "d2h_ms": round(d2h_ms, 3), "d2h_gbs": round(host.d2h_bytes / d2h_ms / 1e6, 2),
            "both_ms": round(both_ms, 3)}


def stored_traffic(elements):
    """DRAM bytes of one bf16 launch from the committed ncu capture of the
    full config-2 launch, scaled to `elements` (traffic grows in proportion
    to the elements decoded); not measured by this run."""
    path = ROOT / "profiles" / "nz_tile_decode_bf16_traffic.txt"
    if not path.is_file():
        return None, None
    fields = {k.strip(): v.strip() for k, v in (line.split("=", 1) for line in path.read_text().splitlines()
                                                if line.startswith(("dram_bytes_per_launch", "elements_per_launch")))}
    if len(fields) != 2:
        return None, None
    per_elem = float(fields["dram_bytes_per_launch"]) / float(fields["elements_per_launch"])
    return int(per_elem * elements), (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one full config-2 bf16 "
                                      f"launch ({path.relative_to(ROOT)}), scaled by elements decoded; "
                                      "not captured in this run")


# ---- bulk decode of one rank's export --------------------------------------------------

def measure_bulk(named, export, args, world, device, clocks):
    """Decodes `export` (one block) once for correctness, then times steps
    of every launch of the block, the dominant launch alone, each dtype
    alone and the host-to-host path. Returns the measurements (times are
    max over ranks)."""
    from neuralzip_b200.gpu.inference import NeuralZipRuntime

    log(f"bulk: upload {len(export.groups)} groups")
    runtime = NeuralZipRuntime(None, export, device)
    block = export.block_order[0]
    batches = runtime._prepared_batches[block]
    decoder = runtime._decoder
    stream = torch.cuda.current_stream(device)

    # Correctness of this very workload before timing: every tensor bit-exact.
    runtime._decode_block(block)
    torch.cuda.synchronize(device)
    views = {}  # one binding per tensor (every group of a tensor names the same one)
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
    main_dtype = main_batch.outputs[0].dtype
    main_groups = [g for g in export.groups if g.encoded.dtype.torch_dtype == main_dtype]
    alg_bytes = algorithmic_bytes(main_groups)
    others = [b for b in batches if b is not main_batch]
    sides = [torch.cuda.Stream(device=device, priority=0) for _ in others]
    fork = torch.cuda.Event()
    joins = [torch.cuda.Event() for _ in others]

    def step(times=None):
        # As nz_decode_launch_many runs them: the big launch first, the
        # others enqueued at once on low-priority streams (they take SMs as
        # its CTAs finish).
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

    log("bulk: bit-exact; timing steps")
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    kernel_events = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    barrier(world)
    with clocks.timed():
        start.record(stream)
        for _ in range(args.steps):
            step(kernel_events)
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    step_ms_rank = start.elapsed_time(end) / args.steps
    step_ms = max_over_ranks(step_ms_rank, world)
    kernel_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kernel_events) / len(kernel_events), world)
    rank_step_ms = gather_over_ranks(step_ms_rank, world)

    # The dominant launch alone (no other launch sharing its tail), after the
    # timed region: the kernel's own rate, beside the in-step one.
    with clocks.timed():
        alone_ms = max_over_ranks(time_launches(lambda: decoder.decode_batch(main_batch, stream), stream,
                                                max(3, min(args.steps, 50)), reps=1), world)

    log("bulk: per-dtype launches")
    # Each dtype's groups in a launch of their own (per-dtype rates).
    per_dtype = {}
    items = runtime._groups_by_block[block]
    for dtype in dict.fromkeys(item.group.encoded.dtype.torch_dtype for item in items):
        mine = [item for item in items if item.group.encoded.dtype.torch_dtype == dtype]
        batch = main_batch if dtype == main_dtype else decoder.prepare_batch([item.device for item in mine])
        for _ in range(3):
            decoder.decode_batch(batch, stream)
        with clocks.timed():
            ms = time_launches(lambda b=batch: decoder.decode_batch(b, stream), stream, 20)
        decoder.check_status(batch)
        ms = max_over_ranks(ms, world)
        groups = [item.group for item in mine]
        nbytes = sum(g.encoded.numel * g.encoded.dtype.element_size for g in groups)
        alg = algorithmic_bytes(groups)
        per_dtype[str(dtype).replace("torch.", "")] = {
            "decoded_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "ms": round(ms, 4), "decoded_bytes": nbytes,
            "algorithmic_gbs": round(alg / (ms * 1e-3) / 1e9, 1), "warps_per_cta": batch.warps_per_cta,
            "ctas": batch.kernel_grid[0], "bit_exact": True}

    e2e = None
    if not args.no_e2e:
        from neuralzip_b200.gpu.bulk import HostDecoder

        log("bulk: e2e (host-to-host)")
        host = HostDecoder(export, device, pieces=args.e2e_pieces)
        for _ in range(max(3, args.warmup // 2)):
            host.decode(stream)
        torch.cuda.synchronize(device)
        barrier(world)
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_steps = max(3, args.steps // 8)
        with clocks.timed():
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
        links = copy_bound(host, stream)
        links["frac"] = round(links["both_ms"] / e_ms, 4)
        links["what"] = ("the step's H2D and D2H bytes copied with no decode, alone and both at once on the "
                         "same streams; frac = both_ms / e2e ms_per_step (1.0: the decode hides entirely "
                         "behind the host copies)")
        e2e = {"value": round(decoded_bytes * world / (e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": host.h2d_bytes, "d2h_bytes_per_step": host.d2h_bytes,
               "ms_per_step": round(e_ms, 3), "copy_bound": links,
               "path": f"HostDecoder: pinned host arena -> H2D -> tile decode -> D2H of every decoded weight, "
                       f"{len(host.pieces)} pieces pipelined on three streams"}
        del host
    result = {"step_ms": step_ms, "kernel_ms": kernel_ms, "alone_ms": alone_ms, "decoded_bytes": decoded_bytes,
              "alg_bytes": alg_bytes, "main_elements": main_batch.elements, "launches": len(batches),
              "per_dtype": per_dtype, "e2e": e2e, "rank_step_ms": rank_step_ms,
              "main_dtype": str(main_dtype).replace("torch.", "")}
    del runtime
    torch.cuda.empty_cache()
    return result


def roofline(m, world):
    peak, peak_kind = peaks()
    achieved = m["alg_bytes"] / (m["kernel_ms"] * 1e-3) / 1e9
    traffic, source = stored_traffic(m["main_elements"])
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
            "frac_of_nominal_8tbs": round(achieved / 8000.0, 4), "traffic": traffic, "traffic_source": source,
            "kernel": f"nz_tile_decode ({m['main_dtype']} launch)", "kernel_ms": round(m["kernel_ms"], 4),
            "algorithmic_bytes": int(m["alg_bytes"]),
            "alone": {"kernel_ms": round(m["alone_ms"], 4),
                      "achieved": round(m["alg_bytes"] / (m["alone_ms"] * 1e-3) / 1e9, 1),
                      "frac": round(m["alg_bytes"] / (m["alone_ms"] * 1e-3) / 1e9 / peak, 4),
                      "note": "the same launch timed by itself after the timed region"}}


# ---- CPU baselines -----------------------------------------------------------------------

def cpu_sample(named, setup, max_chunks):
    """Storage-format frames of up to `max_chunks` mixed-coded bf16 chunks,
    encoded with the reference's own frame encoder; returns ctypes jobs, the
    buffers they point into, and each chunk's codebook (lengths, vocab)."""
    from oracle import oracle as O

    from neuralzip_b200.compressor import NeuralZipCompressor
    from neuralzip_b200.dtypes import DTYPES

    spec = DTYPES[torch.bfloat16]
    comp = NeuralZipCompressor(setup)
    books = {p.codebook_id: p for p in comp.export_codebooks()}
    comp.prepare_storage_transfer_target([(n, t) for n, t in named.items() if t.dtype == torch.bfloat16])
    chunks, keep, decodebooks, chunk_books = [], [], {}, []
    for name, tensor in named.items():
        if tensor.dtype != torch.bfloat16:
            continue
        modes = comp.chunk_modes(name, tensor)
        raw = tensor.reshape(-1).view(torch.uint8).numpy()
        for c, mode in enumerate(modes):
            if mode.kind != "mixed_huffman" or len(chunks) >= max_chunks:
                continue
            part = raw[c * 2 * CHUNK_ELEMS_BF16:(c + 1) * 2 * CHUNK_ELEMS_BF16]
            lanes = O.split(part, spec)
            payload = books[mode.codebook_id]
            lengths = bytes(payload.codebook[4:])
            frame = np.frombuffer(O.ref_mixed_encode_native(lanes[1], lengths, bytes(payload.vocab)), dtype=np.uint8)
            if mode.codebook_id not in decodebooks:
                decodebooks[mode.codebook_id] = O.RefDecodebook(lengths, bytes(payload.vocab))
            out = np.empty(len(part), dtype=np.uint8)
            job = O.RefChunk()
            job.payload, job.payload_size = frame.ctypes.data, len(frame)
            job.book = decodebooks[mode.codebook_id].handle
            job.lanes[0] = lanes[0].ctypes.data
            job.out, job.numel, job.elem_size, job.reorder, job.stream_id = out.ctypes.data, len(lanes[0]), 2, 1, 1
            chunks.append(job)
            keep.append((frame, lanes, out, part))
            chunk_books.append((mode.codebook_id, lengths, bytes(payload.vocab)))
    return chunks, keep, decodebooks, chunk_books


def time_cpu_reference(chunks, keep, chunk_books, seconds_target=10.0, threads=0, cold=False):
    """GB/s of the reference's CPU decode of the sample. cold: every pass
    also builds the decode tables (the reference's make_mixed_table) first,
    as a fresh process would."""
    from oracle import oracle as O

    O.ref_decode_chunks(chunks, threads)  # warm-up + correctness
    for _frame, _lanes, out, part in keep:
        if not np.array_equal(out, part):
            raise AssertionError("reference CPU decode differs from the original chunk")
    decoded = sum(len(part) for *_, part in keep)
    reps, elapsed = 0, 0.0
    start = time.perf_counter()
    while elapsed < seconds_target:
        if cold:
            unique = {cid: (lengths, vocab) for cid, lengths, vocab in chunk_books}
            books = {cid: O.RefDecodebook(lengths, vocab) for cid, (lengths, vocab) in unique.items()}
            for job, (cid, _, _) in zip(chunks, chunk_books):
                job.book = books[cid].handle
        O.ref_decode_chunks(chunks, threads)
        reps += 1
        elapsed = time.perf_counter() - start
    if cold:
        for _frame, _lanes, out, part in keep:
            if not np.array_equal(out, part):
                raise AssertionError("reference CPU decode differs from the original chunk")
    return decoded * reps / elapsed / 1e9, decoded, reps, elapsed


def reference_threads():
    return min(os.cpu_count() or 1, 16)  # the reference pool caps at 16 (common.h:146)


def cpu_baseline_record(named, setup, seconds=10.0):
    """The reference's own CPU decode of mixed bf16 chunks of this workload,
    warm (tables built once) and cold (tables built inside each pass)."""
    from oracle import oracle as O

    if not O.ref_available():
        return None
    log("cpu baseline")
    bf16 = {n: t for n, t in named.items() if t.dtype == torch.bfloat16}
    chunks, keep, books, chunk_books = cpu_sample(bf16, setup, max_chunks=256)
    threads = reference_threads()
    gbs, sample_bytes, reps, elapsed = time_cpu_reference(chunks, keep, chunk_books, seconds, threads)
    cold_gbs, _, cold_reps, cold_elapsed = time_cpu_reference(chunks, keep, chunk_books, seconds / 2, threads,
                                                              cold=True)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
            "cpu_model": cpu_model(), "host_cores": os.cpu_count(),
            "cold": {"value": round(cold_gbs, 3), "reps": cold_reps, "seconds": round(cold_elapsed, 1),
                     "note": "decode tables (make_mixed_table) built inside every pass"},
            "sample": f"{len(chunks)} mixed-coded bf16 chunks ({sample_bytes / 1e6:.0f} MB decoded) x {reps} "
                      f"in {elapsed:.1f} s, reference decode_mixed_block_into + restore_mixed_stream_chunk "
                      "(warm: tables built once)"}


# ---- config 1: one singleton-coded tensor -------------------------------------------------

def config1_record(device, clocks, copies=16, seconds=3.0):
    """Config 1 decode on the GPU (per launch over rotating copies, and all
    copies in one launch) and on the CPU (this build's RFC 8878 4-stream
    Huff0 decoder over the storage format, cold and warm)."""
    from neuralzip_b200.compressor import NeuralZipCompressor
    from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_tensors_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    log("config1: setup")
    named = config1()
    setup = NeuralZipSetup(chunk_size=256 << 10, cluster_js_threshold=0.05, enable_packed_codebooks=False).build(named)
    export = export_tensors_for_gpu(named, setup)
    modes = sorted({g.codebook.vocab == b"" and bool(g.codebook.max_bits) for g in export.groups})
    runtimes = [NeuralZipRuntime(None, export, device) for _ in range(copies)]
    stream = torch.cuda.current_stream(device)
    decoder = runtimes[0]._decoder
    block = export.block_order[0]
    batches = [rt._prepared_batches[block][0] for rt in runtimes]
    for rt in runtimes:
        rt.workspaces[torch.bfloat16].view(torch.uint8).fill_(0xA5)
        rt._decode_block(block)
    torch.cuda.synchronize(device)
    expected = named["w"].reshape(-1).view(torch.uint8)
    for rt in runtimes:
        if not torch.equal(rt.workspaces[torch.bfloat16].view(torch.uint8).cpu(), expected):
            raise AssertionError("config 1 decode is not bit-exact")
        rt.check_status()
    log("config1: bit-exact; graph timing")
    # One decode per launch, cycling over the copies (each copy's inputs and
    # outputs were last touched `copies` launches, ~0.9 GB, earlier: not in
    # L2), replayed from a CUDA graph so host launch cost is not timed.
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device=device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for b in batches:
            decoder.decode_batch(b, side)
    stream.wait_stream(side)
    torch.cuda.synchronize(device)
    with torch.cuda.graph(graph):
        for b in batches:
            decoder.decode_batch(b)
    # Warm-up by time, not count: run alone (--workload config1) this is
    # the process's first GPU work, and a few replays leave the per-launch
    # time at twice its steady value.
    t_warm = time.perf_counter()
    while time.perf_counter() - t_warm < 0.5:
        for _ in range(10):
            graph.replay()
        torch.cuda.synchronize(device)
    with clocks.timed():
        per_launch_ms = time_launches(graph.replay, stream, 10) / copies
    log("config1: batched launch")
    # All copies' groups in one launch (throughput when the GPU is full).
    big = decoder.prepare_batch([item.device for rt in runtimes for item in rt._groups_by_block[block]])
    for _ in range(3):
        decoder.decode_batch(big, stream)
    with clocks.timed():
        big_ms = time_launches(lambda: decoder.decode_batch(big, stream), stream, 20)
    decoder.check_status(big)
    for rt in runtimes:
        if not torch.equal(rt.workspaces[torch.bfloat16].view(torch.uint8).cpu(), expected):
            raise AssertionError("config 1 batched decode is not bit-exact")
    nbytes = named["w"].numel() * 2
    alg = algorithmic_bytes(export.groups)
    warps, ctas = batches[0].warps_per_cta, batches[0].kernel_grid[0]
    peak, peak_kind = peaks()
    del graph, big, runtimes, batches
    torch.cuda.empty_cache()

    # CPU: the storage format (shared_huff0 chunks) decoded by the product's
    # CPU codec, a restatement of RFC 8878's 4-stream Huffman blocks.
    log("config1: CPU decode")
    threads = reference_threads()
    blob, metadata, _storage, _secs = NeuralZipCompressor(setup, threads=threads).encode(named.items())

    def cpu_rate(cold):
        reps, t0 = 0, time.perf_counter()
        warm = NeuralZipCompressor(setup, threads=threads)
        out = warm.decode(blob, metadata)
        if not torch.equal(out["w"].reshape(-1).view(torch.uint8), expected):
            raise AssertionError("CPU decode of config 1 is not bit-exact")
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            comp = NeuralZipCompressor(setup, threads=threads) if cold else warm
            comp.decode(blob, metadata)
            reps += 1
        return nbytes * reps / (time.perf_counter() - t0) / 1e9

    warm_gbs, cold_gbs = cpu_rate(False), cpu_rate(True)
    return {
        "workload": "config1: 4096x4096 bf16 N(0, 0.02), seed 0, 256 KiB chunks, JS 0.05, singleton (Huff0) codebooks",
        "groups": len(export.groups), "singleton_coded": modes == [True], "decoded_bytes": nbytes,
        "per_launch": {"ms": round(per_launch_ms, 4), "decoded_gbs": round(nbytes / (per_launch_ms * 1e-3) / 1e9, 1),
                       "algorithmic_gbs": round(alg / (per_launch_ms * 1e-3) / 1e9, 1),
                       "frac": round(alg / (per_launch_ms * 1e-3) / 1e9 / peak, 4), "peak": peak,
                       "peak_kind": peak_kind, "warps_per_cta": warps, "ctas": ctas,
                       "note": f"one launch per decode of the tensor, {copies} rotating copies (L2 cold), "
                               "replayed from a CUDA graph"},
        "batched": {"copies_per_launch": copies, "ms": round(big_ms, 4),
                    "decoded_gbs": round(copies * nbytes / (big_ms * 1e-3) / 1e9, 1),
                    "frac": round(copies * alg / (big_ms * 1e-3) / 1e9 / peak, 4)},
        "cpu": {"warm_gbs": round(warm_gbs, 3), "cold_gbs": round(cold_gbs, 3), "cores": threads,
                "kind": "port", "cpu_model": cpu_model(),
                "what": "storage v2 shared_huff0 chunks decoded by this build's RFC 8878 4-stream Huffman "
                        "restatement (zstd Huff0 5233c58 is absent); cold = fresh decoder (tables built) per pass"},
        "bit_exact": True,
    }


# ---- configs 3 and 4: batch-1 greedy generation -------------------------------------

def _model_config(name):
    from transformers import LlamaConfig, Qwen2Config

    if name == "config3":  # Qwen2.5-0.5B architecture
        return Qwen2Config(hidden_size=896, num_hidden_layers=24, num_attention_heads=14, num_key_value_heads=2,
                           intermediate_size=4864, vocab_size=151936, tie_word_embeddings=True,
                           max_position_embeddings=4096), 32, 128
    if name == "config5b":  # Llama-3-70B architecture
        return LlamaConfig(hidden_size=8192, num_hidden_layers=80, num_attention_heads=64, num_key_value_heads=8,
                           intermediate_size=28672, vocab_size=128256, max_position_embeddings=4096), 128, 64
    return LlamaConfig(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                       intermediate_size=14336, vocab_size=128256, max_position_embeddings=4096), 128, 256


def _busy_us(events):
    """Union length (us) of device-side intervals."""
    total, cur_s, cur_e = 0.0, None, None
    for s, e in sorted(events):
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                total += cur_e - cur_s
            cur_s, cur_e = s, e
        else:
            cur_e = max(cur_e, e)
    if cur_e is not None:
        total += cur_e - cur_s
    return total


def gpu_busy_ms_per_token(run, n):
    """GPU-busy ms per generated token: the union of the device intervals
    (kernels, copies, sets) recorded by torch.profiler (CUPTI) during a
    generation of n + 1 tokens minus one of 1 token, over n. Busy time, not
    wall time: gaps where the GPU waits for the host are excluded."""
    from torch.autograd import DeviceType
    from torch.profiler import ProfilerActivity, profile

    def busy(k):
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            run(k)
            torch.cuda.synchronize()
        spans = [(e.time_range.start, e.time_range.end) for e in prof.events() if e.device_type == DeviceType.CUDA]
        return _busy_us(spans), sum(b - a for a, b in spans)

    full, full_sum = busy(n + 1)
    one, one_sum = busy(1)
    return (full - one) / n / 1e3, (full_sum - one_sum) / n / 1e3


def checkpoint_v3_record(model, setup, prompt, uncompressed, device):
    """save_pretrained of the compressed model (its weights materialized
    from the GPU, storage v2 encoded on the host) and from_pretrained of the
    v3 checkpoint (decoded on the host, exported and attached again). The
    reloaded weights must equal the uncompressed model's bit for bit, and
    its first-step logits must equal those of the same weights loaded by
    Transformers' own from_pretrained from an ordinary checkpoint (both
    loads with the same dtype and attention, so both models are built the
    same way)."""
    import tempfile

    from neuralzip_b200 import neuralzip
    from neuralzip_b200.gpu import pretrained

    neuralzip(setup, device=device)
    cls = type(uncompressed)
    options = {"dtype": torch.bfloat16, "attn_implementation": "eager"}
    with tempfile.TemporaryDirectory() as folder:
        compressed_dir, plain_dir = Path(folder) / "v3", Path(folder) / "plain"
        t0 = time.perf_counter()
        model.save_pretrained(compressed_dir)
        save_s = time.perf_counter() - t0
        stored = model.neuralzip_stats
        size = sum(f.stat().st_size for f in compressed_dir.iterdir())
        t0 = time.perf_counter()
        loaded = cls.from_pretrained(compressed_dir, **options)
        torch.cuda.synchronize(device)
        load_s = time.perf_counter() - t0
        pretrained._ORIGINAL["save"](uncompressed, plain_dir)
        reference = pretrained._ORIGINAL["load"](cls, plain_dir, **options).to(device).eval()
    original = uncompressed.state_dict()
    weights_identical = all(torch.equal(w.view(torch.uint8), original[name].cpu().view(torch.uint8))
                            for name, w in loaded.neuralzip_runtime.materialized_weights())
    stats = loaded.neuralzip_stats
    with torch.no_grad():
        logits = loaded(prompt, use_cache=False).logits.float().cpu()
        want = reference(prompt, use_cache=False).logits.float().cpu()
    identical = bool(torch.equal(logits.view(torch.int32), want.view(torch.int32)))
    del loaded, reference
    if not (weights_identical and identical):
        raise AssertionError(f"v3 reload differs: weights {weights_identical}, logits {identical}")
    return {"save_s": round(save_s, 2), "load_s": round(load_s, 2), "checkpoint_bytes": size,
            "storage_ratio": round(stored.compression_ratio, 4),
            "decoding_seconds": round(stats.decoding_seconds, 3),
            "runtime_encoding_seconds": round(stats.runtime_encoding_seconds, 3),
            "weights_bitwise": weights_identical, "first_step_logits_bitwise": identical,
            "what": "save_pretrained (GPU materialize + host storage encode + safetensors write), then "
                    "from_pretrained (host storage decode + model build + GPU export + attach); logits "
                    "compared with the same weights loaded by Transformers from an ordinary checkpoint"}


def static_decoder(m, prompt, new_tokens, device):
    """Greedy decoding of `prompt` with a static KV cache, as graph_decode
    captures it: the prefill runs (eagerly) here, and returns the first
    token, `step()` (one token: the model on the current ids with the
    position, the causal mask and each cache layer's length counter all on
    the device, its argmax written back to the ids) and `rewind()` (back to
    the state right after the prefill)."""
    from transformers import StaticCache

    _batch, plen = prompt.shape
    length = plen + new_tokens + 4
    cache = StaticCache(config=m.config, max_cache_len=length)
    first = m(input_ids=prompt, past_key_values=cache, use_cache=True).logits[:, -1].argmax(-1)
    ids = first[:, None].clone()
    pos = torch.full((1,), plen, dtype=torch.long, device=device)
    kv = torch.arange(length, device=device)
    low = torch.finfo(torch.bfloat16).min

    def step():
        # A 4D mask is used as given, so nothing is built on the host.
        mask = ((kv > pos).to(torch.bfloat16) * low).view(1, 1, 1, length)
        nxt = m(input_ids=ids, past_key_values=cache, position_ids=pos.view(1, 1), attention_mask=mask,
                use_cache=True).logits[:, -1].argmax(-1)
        ids.copy_(nxt[:, None])
        pos.add_(1)
        return nxt

    def rewind():
        for layer in cache.layers:
            layer.cumulative_length.fill_(plen)
        ids.copy_(first[:, None])
        pos.fill_(plen)

    return first, step, rewind


def graph_decode(m, prompt, new_tokens, device, reps):
    """Greedy decoding of `new_tokens` after `prompt` with the one-token
    step of static_decoder captured once in a CUDA graph, so no host work
    is timed: the prefill runs eagerly (not timed), then every step is one
    replay (the graph feeds its argmax token and position back to its
    inputs). Returns the tokens and the ms per token of each rep (CUDA
    events over the replays). With a compressed model the capture holds the
    decode launches its forward pre-hooks enqueue, side-stream prefetches
    included."""
    stream = torch.cuda.current_stream(device)
    with torch.no_grad():
        first, step, rewind = static_decoder(m, prompt, new_tokens, device)
        # Warm-up on a side stream before the capture (positions the timed
        # replays rewrite; later positions are masked until written).
        side = torch.cuda.Stream(device=device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        stream.wait_stream(side)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            nxt = step()
        times, tokens = [], None
        for _ in range(reps):
            rewind()
            steps = []
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(new_tokens - 1):
                graph.replay()
                steps.append(nxt.clone())
            b.record(stream)
            torch.cuda.synchronize(device)
            times.append(a.elapsed_time(b) / (new_tokens - 1))
            tokens = torch.cat([first[:, None], torch.stack(steps, 1)], 1)
        del graph
    return tokens, times


def graph_record(model, uncompressed, prompt, new_tokens, device, reps):
    """Both models decoded by graph_decode, alternately; the tokens must be
    identical (asserted)."""
    ref_ms, comp_ms = [], []
    for _ in range(reps):
        ref_tokens, t = graph_decode(uncompressed, prompt, new_tokens, device, 1)
        ref_ms += t
        tokens, t = graph_decode(model, prompt, new_tokens, device, 1)
        comp_ms += t
    if not torch.equal(tokens, ref_tokens):
        raise AssertionError("CUDA-graph generation of the compressed model differs from the uncompressed model")
    batch = prompt.shape[0]
    ref, comp = statistics.median(ref_ms), statistics.median(comp_ms)
    return {"tok_s": round(batch / (comp * 1e-3), 3), "uncompressed_tok_s": round(batch / (ref * 1e-3), 3),
            "ratio_vs_uncompressed": round(ref / comp, 4), "ms_per_token": round(comp, 3),
            "uncompressed_ms_per_token": round(ref, 3), "tokens_identical": True,
            "timing": "static KV cache, the one-token step captured once in a CUDA graph (decode launches and "
                      f"side-stream prefetches of the compressed model included); CUDA events over {new_tokens - 1} "
                      f"replays, median of {reps} runs alternating with the uncompressed model"}


def generation_record(workload, device, *, batch=1, new_tokens=None, reps=3, overlap=True, prefetch_depth=2,
                      blocks_per_launch=0, tp=None, busy_tokens=16, v3=False, layers=None, graphs=False):
    """Random-init model of the config's architecture (N(0, 0.02), norms 1),
    compressed through neuralzip.setup + the GPU export, then greedy
    generation with KV cache and eager attention. An uncompressed copy of
    the same model is timed alternately with the compressed one (medians of
    `reps` runs each, so drift of the host or the GPU hits both alike); both
    must generate the same tokens, and the first-step logits must be equal
    bit for bit (asserted)."""
    import copy

    from transformers import AutoModelForCausalLM

    from neuralzip_b200.gpu.inference import NeuralZipRuntime, export_model_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    torch.cuda.set_device(device)
    config, prompt_len, default_tokens = _model_config(workload)
    if layers:
        config.num_hidden_layers = int(layers)
    new_tokens = new_tokens or default_tokens
    config._attn_implementation = "eager"  # the reference's GPU protocol (eager attention)
    torch.manual_seed(0)
    if workload == "config5b":  # each rank builds only its slices (and its replicated parts)
        from transformers import LlamaForCausalLM

        from neuralzip_b200.gpu.tp import build_tensor_parallel

        rank, world = tp if tp is not None else (0, 1)
        model, _hooks = build_tensor_parallel(LlamaForCausalLM, config, rank, world, dtype=torch.bfloat16,
                                              device=device)
        tp = None  # already sliced
        sliced = True
    else:
        sliced = False
        with torch.device(device):
            model = AutoModelForCausalLM.from_config(config, dtype=torch.bfloat16).eval()
    prompt = torch.randint(config.vocab_size, (batch, prompt_len),
                           generator=torch.Generator().manual_seed(1)).to(device)

    def runner(m):
        def run(n):
            with torch.no_grad():
                return m.generate(prompt, max_new_tokens=n, min_new_tokens=n, do_sample=False, use_cache=True,
                                  pad_token_id=0)
        return run

    def generate(m):
        """Tokens and seconds per generation step after the first (prefill
        and per-call setup excluded by timing a one-token call too)."""
        run = runner(m)
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        out = run(new_tokens)
        torch.cuda.synchronize(device)
        full = time.perf_counter() - t0
        t0 = time.perf_counter()
        run(1)
        torch.cuda.synchronize(device)
        one = time.perf_counter() - t0
        return out, (full - one) / (new_tokens - 1)

    if tp is not None:  # tensor parallel: each rank keeps and compresses its slices
        from neuralzip_b200.gpu.tp import shard_for_tensor_parallel

        shard_for_tensor_parallel(model, *tp)
        torch.cuda.empty_cache()
    with torch.no_grad():
        ref_logits = model(prompt, use_cache=False).logits.float().cpu()
    uncompressed = copy.deepcopy(model)
    log(f"generation: {workload} setup")
    t0 = time.perf_counter()
    setup = NeuralZipSetup().build(model)
    exported = export_model_for_gpu(model, setup)
    prep_s = time.perf_counter() - t0
    per_launch = "auto" if blocks_per_launch == 0 else blocks_per_launch
    runtime = NeuralZipRuntime.attach(model, exported, device=device, overlap=overlap,
                                      prefetch_depth=prefetch_depth, blocks_per_launch=per_launch)
    with torch.no_grad():
        logits = model(prompt, use_cache=False).logits.float().cpu()
    identical = bool(torch.equal(logits.view(torch.int32), ref_logits.view(torch.int32)))
    log("generation: timing")
    generate(uncompressed)  # warm-up
    generate(model)
    ref_times, comp_times = [], []
    for _ in range(reps):
        ref_tokens, t = generate(uncompressed)
        ref_times.append(t)
        tokens, t = generate(model)
        comp_times.append(t)
    tokens_identical = bool(torch.equal(tokens, ref_tokens))
    busy = {}
    log("generation: GPU-busy (torch.profiler)")
    for name, m in (() if sliced else (("uncompressed", uncompressed), ("compressed", model))):
        try:
            union, total = gpu_busy_ms_per_token(runner(m), busy_tokens)
            busy[name] = {"busy_ms_per_token": round(union, 3), "kernel_sum_ms_per_token": round(total, 3)}
        except Exception as exc:  # the profiler is evidence, not the measurement
            busy[name] = {"error": f"{type(exc).__name__}: {exc}"[:200]}
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
    runtime.check_status()
    graph = None
    if graphs:
        log("generation: CUDA-graph mode")
        try:
            graph = graph_record(model, uncompressed, prompt, new_tokens, device, reps)
        except AssertionError:
            raise
        except Exception as exc:  # a capture the library or Transformers refuses is reported, not hidden
            graph = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    checkpoint = checkpoint_v3_record(model, setup, prompt, uncompressed, device) if v3 else None
    decoded = sum(g.encoded.numel * g.encoded.dtype.element_size for g in exported.groups)
    ref_s, comp_s = statistics.median(ref_times), statistics.median(comp_times)
    record = {
        "workload": workload, "batch": batch, "prompt": prompt_len, "new_tokens": new_tokens,
        "tok_s": round(batch / comp_s, 3), "uncompressed_tok_s": round(batch / ref_s, 3),
        "ratio_vs_uncompressed": round(ref_s / comp_s, 4),
        "ratio_runs": [round(r / c, 4) for r, c in zip(ref_times, comp_times)],
        "tokens_identical": tokens_identical, "first_step_logits_bitwise": identical,
        "gpu_busy": busy, "overlap": runtime.overlap, "prefetch_depth": runtime.prefetch_depth,
        "blocks_per_launch": runtime.blocks_per_launch, "launch_units": len(runtime._units),
        "decode_per_step_ms": round(min(decode_ms), 3),
        "decode_gbs": round(decoded / (min(decode_ms) * 1e-3) / 1e9, 1), "decoded_bytes_per_step": decoded,
        "compressed_weights": len({b.tensor_name for b in exported.bindings}), "prep_s": round(prep_s, 1),
        "attn": "eager", "kv_cache": True,
        "timing": "(t(new_tokens) - t(1)) / (new_tokens - 1): prefill excluded; "
                  f"median of {reps} runs alternating with the uncompressed model",
    }
    if checkpoint is not None:
        record["checkpoint_v3"] = checkpoint
    if graph is not None:
        record["cuda_graph"] = graph
    if not (tokens_identical and identical):
        raise AssertionError(f"compressed generation differs from the uncompressed model: {record}")
    del runtime, model, uncompressed
    torch.cuda.empty_cache()
    return record, tokens, ref_s, comp_s


def run_generation(args, world, rank, local):
    """--workload config3|config4|config5b: the generation record as its own line."""
    device = torch.device("cuda", local)
    tp = (rank, world) if (args.tp or args.workload == "config5b") and world > 1 else None
    record, tokens, ref_s, comp_s = generation_record(
        args.workload, device, batch=args.batch, new_tokens=args.new_tokens, reps=args.gen_reps,
        overlap=not args.no_overlap, prefetch_depth=args.prefetch_depth,
        blocks_per_launch=args.blocks_per_launch, tp=tp, layers=args.layers,
        graphs=args.cuda_graphs and tp is None)
    if tp is not None:
        from neuralzip_b200.gpu.tp import assert_same_on_all_ranks

        assert_same_on_all_ranks(tokens)
        ref_s, comp_s = max_over_ranks(ref_s, world), max_over_ranks(comp_s, world)
        record["tok_s"], record["uncompressed_tok_s"] = round(args.batch / comp_s, 3), round(args.batch / ref_s, 3)
        record["ratio_vs_uncompressed"] = round(ref_s / comp_s, 4)
    if rank == 0:
        print(json.dumps({
            "metric": f"batch-{args.batch} greedy generation tok/s, compressed weights decoded per layer per step",
            "value": record["tok_s"], "unit": "tok/s", "n_gpus": world if tp else 1, "higher_is_better": True,
            "parallelism": f"tp{world}, NCCL all-reduce after o_proj and down_proj" if tp else "single GPU",
            **record}))


def run_config1(local):
    """--workload config1: the config-1 record (one 4096x4096 bf16 tensor,
    singleton codebooks) as its own line, on one GPU."""
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    with NvmlClocks(device.index) as clocks:
        record = config1_record(device, clocks)
    print(json.dumps({
        "metric": "decoded weight GB/s (config 1, one decode per launch)",
        "value": record["per_launch"]["decoded_gbs"], "unit": "GB/s", "n_gpus": 1, "higher_is_better": True,
        "clocks": clocks.summary(), **record}))


# ---- --impl reference -------------------------------------------------------------

def run_reference(args, world, rank):
    """--impl reference: the reference's CPU decode on the host cores, on a
    bounded sample of the same workload's mixed-coded bf16 chunks."""
    if rank != 0:
        return
    from oracle import oracle as O

    from neuralzip_b200.setup import NeuralZipSetup

    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (reference sources absent)"}))
        return
    if world > 1:
        share = config5a_share(world * args.layers_per_gpu, 0, world)
        named = {k: v for k, v in config5a_generate(share, torch.device("cuda", 0)).items()}
        workload = "config5a-bf16-mixed-sample"
    else:
        named = {n: t for n, t in config2(1, args.bf16_tensors).items() if t.dtype == torch.bfloat16}
        workload = "config2-bf16-mixed-sample"
    setup = NeuralZipSetup().build(named)
    chunks, keep, _books, _chunk_books = cpu_sample(named, setup, max_chunks=512)
    threads = reference_threads()
    O.ref_decode_chunks(chunks, threads)
    for _frame, _lanes, out, part in keep:
        if not np.array_equal(out, part):
            raise AssertionError("reference CPU decode differs from the original chunk")
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
    sample = (f"{len(chunks)} mixed-coded bf16 chunks of {workload.split('-')[0]}, {decoded / 1e6:.0f} MB decoded "
              "per step, storage-format frames from the reference encoder")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": workload, "chunks": len(chunks), "threads": threads,
                   "untimed": "codebooks chosen by this build's NeuralZipSetup (the reference's setup decisions) "
                              "and chunks encoded by the reference's own encoder, before the timed decode"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "cpu_model": cpu_model(), "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---- main ----------------------------------------------------------------------------

def config5a_record(args, world, rank, device, clocks, host_threads, layers_per_gpu):
    """Config 5a: this rank's byte-balanced share of a world x
    layers_per_gpu layer checkpoint, generated, compressed and decoded here."""
    from neuralzip_b200.gpu.inference import export_tensors_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    log("config5a: generate")
    t0 = time.perf_counter()
    share = config5a_share(world * layers_per_gpu, rank, world)
    named = config5a_generate(share, device)
    t_gen = time.perf_counter() - t0
    log("config5a: setup")
    setup = NeuralZipSetup().build(named)
    t_setup = time.perf_counter() - t0 - t_gen
    export = export_tensors_for_gpu(named, setup, threads=host_threads)
    t_export = time.perf_counter() - t0 - t_gen - t_setup
    m = measure_bulk(named, export, args, world, device, clocks)
    m["config"] = {"workload": "config5a", "layers": world * layers_per_gpu, "layers_per_gpu": layers_per_gpu,
                   "tensors_this_rank": len(named), "groups_this_rank": len(export.groups),
                   "decoded_bytes_per_gpu": m["decoded_bytes"],
                   "codebooks": sorted({(b.mode, len(b.vocab) // 2) for b in setup.codebooks}),
                   "generate_s": round(t_gen, 1), "setup_s": round(t_setup, 1), "export_s": round(t_export, 1),
                   "partition": "contiguous 256 KiB chunk ranges balanced by decoded bytes "
                                "(neuralzip_b200.gpu.shard.partition rule); each rank generates only its range",
                   "l2": "inputs and outputs larger than L2 (no flush)"}
    return m


def main():
    args = parse_args()
    world, rank, local = dist_setup()
    if args.workload != "bulk" or args.impl == "reference":
        if args.workload == "config1":
            run_config1(local)
        elif args.workload != "bulk":
            run_generation(args, world, rank, local)
        else:
            run_reference(args, world, rank)
        barrier(world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    from neuralzip_b200.gpu.inference import export_tensors_for_gpu
    from neuralzip_b200.setup import NeuralZipSetup

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    # Ranks share the host: each builds its workload on its share of the cores.
    host_threads = max(1, (os.cpu_count() or 1) // world)
    if world > 1:
        torch.set_num_threads(host_threads)
    with NvmlClocks(device.index) as clocks:
        extras = {}
        if world == 1:
            log("config2: generate + setup")
            t0 = time.perf_counter()
            named = config2(1, args.bf16_tensors)
            setup = NeuralZipSetup().build(named)
            t_setup = time.perf_counter() - t0
            export = export_tensors_for_gpu(named, setup, threads=host_threads)
            t_export = time.perf_counter() - t0 - t_setup
            m = measure_bulk(named, export, args, world, device, clocks)
            config = {"workload": "config2", "bf16_tensors": args.bf16_tensors, "decoded_bytes_per_gpu": m["decoded_bytes"],
                      "groups": len(export.groups), "launches_per_step": m["launches"],
                      "codebooks": sorted({(b.mode, len(b.vocab) // 2) for b in setup.codebooks}),
                      "l2": "inputs and outputs larger than L2 (no flush)", "setup_s": round(t_setup, 1),
                      "export_s": round(t_export, 1), "parallelism": "1 GPU", "host_cores": os.cpu_count()}
            cpu = None if args.no_cpu_baseline else cpu_baseline_record(named, setup)
            del named, setup, export
            if not args.no_config1:
                extras["config1"] = config1_record(device, clocks)
            if not args.no_config5a:
                m5 = config5a_record(args, 1, 0, device, clocks, host_threads, args.layers_per_gpu)
                extras["config5a_1gpu"] = {
                    "value": round(m5["decoded_bytes"] / (m5["step_ms"] * 1e-3) / 1e9, 3), "unit": "GB/s",
                    "ms_per_step": round(m5["step_ms"], 4), "roofline": roofline(m5, 1),
                    "per_dtype": m5["per_dtype"], "config": m5["config"],
                    "note": "one GPU's share of the multi-GPU workload (what each rank decodes under torchrun)"}
            if not args.no_generation:
                log("generation: config3")
                record, *_ = generation_record("config3", device, v3=True, graphs=True)
                extras["generation"] = record
        else:
            m = config5a_record(args, world, rank, device, clocks, host_threads, args.layers_per_gpu)
            config = dict(m["config"], parallelism=f"{world} ranks, disjoint chunk ranges, no collective",
                          host_cores=os.cpu_count(), host_threads_per_rank=host_threads)
            cpu = None
    clock = clocks.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(m["decoded_bytes"] * world / (m["step_ms"] * 1e-3) / 1e9, 3),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": round(m["step_ms"], 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic", "config": config,
            "roofline": roofline(m, world), "per_dtype": m["per_dtype"], "cpu_baseline": cpu, "e2e": m["e2e"],
            "clocks": clock, "gpu_launches": args.steps * m["launches"],
        }
        if world > 1:
            line["rank_step_ms"] = [round(x, 4) for x in m["rank_step_ms"]]
            line["limiter"] = ("slowest rank's decode step (max over ranks); spread "
                               f"{(max(m['rank_step_ms']) - min(m['rank_step_ms'])) / min(m['rank_step_ms']):.2%}")
        line.update(extras)
        print(json.dumps(line))
    barrier(world)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
