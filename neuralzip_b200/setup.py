"""Offline setup: chunk clustering and codebook learning.

Public surface of neuralzip/setup.py:21-89 (``NeuralZipSetup`` with the same
constructor options, pickle fields, ``build``/``save``/``load`` and
``setup_seconds``) and the same decisions:

* every floating tensor's coded byte lane is cut into ``chunk_size``-byte
  source chunks, and each chunk's exponent distribution is clustered with
  the chunks before it (same dtype and forced label; nearest centroid by
  base-2 Jensen-Shannon distance, joined when within
  ``cluster_js_threshold``), keeping up to ``max_codebook_sample_bytes`` of
  sample bytes per cluster;
* each cluster gets a singleton (Huff0) table and, where the dtype has a
  pure exponent lane, an adaptive pair/singleton ("mixed") table with up to
  254 pairs, pruned until every pair codes no longer than its two halves,
  and kept when its estimated stored size on up to four sample chunks beats
  the singleton's;
* every (tensor, dtype, lane) also gets a pooled singleton table, for
  tensors whose shape differs at transfer time.

The design differs from the reference's: histograms, lane splits and token
counts are native passes over whole tensors; the clustering is one native
pass over all chunks (``nz_cluster_chunks``); and the two table options are
sized with measure-only encodes of the sample lanes under the packer's own
raw-fallback rule, instead of six timed storage compressions of rebuilt
element data.
"""

from __future__ import annotations

import pickle
import time
from dataclasses import dataclass
from pathlib import Path
from statistics import median

import numpy as np
import torch

from neuralzip_b200 import _native, huff0
from neuralzip_b200.dtypes import DTYPES
from neuralzip_b200.payloads import CHUNK_METADATA_BYTES, CodebookPayload
from neuralzip_b200.utils import _floating_tensors, _model_tensors, _stream_chunk_size, time_call

MAX_PAIRS = 254
CODED_METADATA = CHUNK_METADATA_BYTES["shared_huff0"]
RAW_METADATA = CHUNK_METADATA_BYTES["raw"]


@dataclass(frozen=True)
class NeuralZipSetupReport:
    clustering_seconds: float
    codebook_setup_seconds: float

    @property
    def setup_seconds(self):
        return self.clustering_seconds + self.codebook_setup_seconds


@dataclass
class _Cluster:
    dtype: str
    lane: int
    weight: int = 0          # source bytes of the cluster's chunks
    sampled: int = 0
    samples: list = None

    def __post_init__(self):
        self.samples = []


def _dtype_struct(spec):
    return _native.dtype_struct(spec.element_size, spec.bit_reorder, spec.mantissa_bits, spec.exponent_bits,
                                spec.gpu_stream)


class NeuralZipSetup:
    def __init__(
        self, *, min_saving_bytes=0, chunk_size=256 << 10,
        compression_threshold=0.95, prior_count=1, cluster_map=None,
        cluster_js_threshold=0.05, max_codebook_sample_bytes=8 << 20,
        enable_shared_codebooks=True, enable_packed_codebooks=True,
    ):
        if chunk_size < 4 or max_codebook_sample_bytes < 1 or prior_count < 1:
            raise ValueError("Chunk size >= 4, sample budget >= 1, and prior >= 1 are required.")
        self.min_saving_bytes = int(min_saving_bytes)
        self.chunk_size = int(chunk_size)
        self.compression_threshold = float(compression_threshold)
        self.prior_count = int(prior_count)
        self.cluster_map = dict(cluster_map or {})
        self.cluster_js_threshold = float(cluster_js_threshold)
        self.max_codebook_sample_bytes = int(max_codebook_sample_bytes)
        self.enable_shared_codebooks = bool(enable_shared_codebooks)
        self.enable_packed_codebooks = bool(enable_packed_codebooks)
        self.codebooks = ()
        self.chunk_codebooks = {}
        self.tensor_codebooks = {}
        self.global_codebooks = {}
        self.packing_report = ()
        self.setup_report = NeuralZipSetupReport(0.0, 0.0)

    @property
    def setup_seconds(self):
        return self.setup_report.setup_seconds

    @property
    def _coding(self):
        return self.enable_shared_codebooks or self.enable_packed_codebooks

    def build(self, model):
        (clusters, assignments, pooled), clustering_seconds = time_call(self._cluster, _model_tensors(model))
        (books, chunks, tensors, report), codebook_seconds = time_call(
            self._codebooks_for, clusters, assignments, pooled)
        self.codebooks = tuple(books)
        self.chunk_codebooks = chunks
        self.tensor_codebooks = tensors
        self.global_codebooks = {}
        self.packing_report = tuple(report)
        self.setup_report = NeuralZipSetupReport(clustering_seconds, codebook_seconds)
        return self

    def save(self, path):
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        with path.open("wb") as handle:
            pickle.dump(self, handle, protocol=5)
        return path

    @classmethod
    def load(cls, value):
        if not isinstance(value, cls):
            with Path(value).open("rb") as handle:
                value = pickle.load(handle)
        if not isinstance(value, cls) or not hasattr(value, "chunk_codebooks"):
            raise TypeError("Expected a current chunk-level NeuralZip setup.")
        return value

    # ---- clustering -------------------------------------------------------------

    def _cluster(self, named_tensors):
        """(clusters, {(name, dtype, lane, numel): cluster per chunk},
        {(name, dtype, lane): pooled byte counts})."""
        lanes, keys, pooled = [], [], {}
        distributions, weights, classes, forced = [], [], [], []
        class_ids = {}
        for name, tensor in _floating_tensors(named_tensors):
            spec = DTYPES[tensor.dtype]
            raw = tensor.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy()
            dt = _dtype_struct(spec)
            lane = _native.split_lanes(raw, dt, selected_only=True)[spec.gpu_stream]
            step = _stream_chunk_size(self.chunk_size, spec.element_size)
            key = (str(name), spec.name, spec.gpu_stream)
            pooled[key] = _native.count_tokens(lane, b"")
            counts = _native.exponent_histograms(raw, dt, step).astype(np.float64)
            distributions.append(counts / counts.sum(axis=1, keepdims=True))
            starts = range(0, len(lane), step)
            weights.extend(min(step, len(lane) - s) for s in starts)
            for index in range(len(starts)):
                label = self.cluster_map.get((name, index), self.cluster_map.get(name))
                classes.append(class_ids.setdefault((spec.name, label), len(class_ids)))
                forced.append(label is not None)
            lanes.append((lane, step))
            keys.append((*key, tensor.numel()))
        if not keys:
            return [], {}, pooled
        assign, _centroids = _native.cluster_chunks(
            np.concatenate(distributions), weights, classes, forced, self.cluster_js_threshold,
            share=self.enable_shared_codebooks)
        clusters = {}
        assignments = {}
        position = 0
        for key, (lane, step) in zip(keys, lanes):
            ids = []
            for start in range(0, len(lane), step):
                cid = int(assign[position])
                position += 1
                cluster = clusters.setdefault(cid, _Cluster(key[1], key[2]))
                part = lane[start:start + step]
                cluster.weight += len(part)
                take = self.max_codebook_sample_bytes - cluster.sampled
                if take > 0:
                    sample = part[:take].tobytes()
                    cluster.samples.append(sample)
                    cluster.sampled += len(sample)
                ids.append(cid)
            assignments[key] = tuple(ids)
        return [clusters[i] for i in range(len(clusters))], assignments, pooled

    # ---- codebooks --------------------------------------------------------------

    def _codebooks_for(self, clusters, assignments, pooled):
        books, index, report = [], {}, []

        def register(book, dtype, lane, vocab=b""):
            if book is None or not self._coding:
                return None
            mode = "mixed_huffman" if vocab else "shared_huff0"
            key = (dtype, lane, mode, book.codebook, vocab)
            if not self.enable_shared_codebooks:
                key += (len(books),)
            if key not in index:
                index[key] = len(books)
                books.append(CodebookPayload(len(books), lane, dtype, mode, book.codebook, vocab=vocab))
            return index[key]

        specs = {spec.name: spec for spec in DTYPES.values()}
        per_cluster = []
        for number, cluster in enumerate(clusters):
            book, vocab, scores = self._cluster_codebook(cluster, specs[cluster.dtype])
            if scores is not None:
                report.append({"cluster": number, **scores})
            per_cluster.append(register(book, cluster.dtype, cluster.lane, vocab))
        chunks = {key: tuple(per_cluster[c] for c in ids) for key, ids in assignments.items()}
        tensors = {key: register(self._singleton(counts), key[1], key[2]) for key, counts in pooled.items()}
        return books, chunks, tensors, report

    def _singleton(self, counts):
        if not self._coding:
            return None
        try:
            return huff0.build_codebook_from_counts(counts, prior_count=self.prior_count, max_bits=12)
        except RuntimeError:
            return None  # some uniform alphabets have no serializable table: stored raw

    def _cluster_codebook(self, cluster, spec):
        """(table, pair vocabulary, comparison report or None)."""
        if not self._coding:
            return None, b"", None
        singleton = self._singleton(huff0.count_mixed_tokens(cluster.samples, b""))
        if not self.enable_packed_codebooks or spec.exponent_stream is None:
            return singleton, b"", None
        # Adjacent-byte pairs inside each sample, the most frequent first
        # (stable on ties), at most MAX_PAIRS, in pair-value order.
        pairs = np.zeros(1 << 16, dtype=np.int64)
        for sample in cluster.samples:
            b = np.frombuffer(sample, dtype=np.uint8).astype(np.uint32)
            pairs += np.bincount(b[:-1] | (b[1:] << 8), minlength=1 << 16)
        seen = np.flatnonzero(pairs)
        chosen = np.sort(seen[np.argsort(-pairs[seen], kind="stable")[:MAX_PAIRS]]).astype("<u2")
        candidates = len(chosen)
        # Drop every pair whose code is longer than its halves' codes and
        # rebuild, until all pairs pay for themselves.
        while len(chosen):
            vocab = chosen.tobytes()
            mixed = huff0.build_mixed_codebook(huff0.count_mixed_tokens(cluster.samples, vocab), vocab,
                                               prior_count=self.prior_count)
            lengths = np.frombuffer(mixed.codebook[4:], dtype=np.uint8).astype(np.uint16)
            worth = lengths[256:] <= lengths[chosen & 255] + lengths[chosen >> 8]
            if worth.all():
                scores = self._size_options(cluster, spec, singleton, mixed, vocab)
                scores.update(candidate_pairs=candidates, kept_pairs=len(chosen))
                return (mixed, vocab, scores) if scores["mode"] == "mixed_huffman" else (singleton, b"", scores)
            chosen = chosen[worth]
        return singleton, b"", None

    def _stored_size(self, kind, book, lane):
        """(stored bytes incl. chunk metadata, coded?) of one source chunk's
        lane under the packer's rule (huff0.compress_direct_storage): coded
        when the payload fits the budget and saves enough, else raw."""
        length = len(lane)
        budget = int(length * self.compression_threshold) - CODED_METADATA
        payload = 0
        if budget > 0 and kind == "shared_huff0" and length <= huff0.MAX_BLOCK_SIZE:
            payload = _native.huff0_encode(book.handle, lane, length, measure=True)
            payload = payload if payload <= budget else 0
        elif budget > 0 and kind == "mixed_huffman":
            payload = _native.mixed_encode(book.handle, lane, budget, measure=True)
        if payload and payload + self.min_saving_bytes < length and \
                payload + CODED_METADATA < length * self.compression_threshold:
            return payload + CODED_METADATA, True
        return length + RAW_METADATA, False

    def _size_options(self, cluster, spec, singleton, mixed, vocab):
        """Estimated stored bytes of the cluster under each table, from up to
        four sample chunks spread over its samples, scaled to the cluster's
        bytes, plus the table's own metadata when a chunk would use it."""
        pick = np.linspace(0, len(cluster.samples) - 1, min(4, len(cluster.samples)), dtype=int)
        lanes = [np.frombuffer(cluster.samples[i], dtype=np.uint8) for i in pick]
        sampled = sum(len(lane) for lane in lanes)
        options = (("shared_huff0" if singleton is not None else "raw", singleton, b""),
                   ("mixed_huffman", mixed, vocab))
        sizes, seconds = [], []
        for kind, book, option_vocab in options:
            runs = []
            for _ in range(3):
                t0 = time.perf_counter()
                measured = [self._stored_size(kind, book, lane) for lane in lanes]
                runs.append(time.perf_counter() - t0)
            stored = sum(size for size, _ in measured)
            used = any(coded for _, coded in measured)
            table = CodebookPayload(0, cluster.lane, spec.name, kind, book.codebook, vocab=option_vocab).metadata_bytes \
                if book is not None and used else 0
            sizes.append(stored * cluster.weight / sampled + table)
            seconds.append(median(runs))
        mode = "mixed_huffman" if sizes[1] < sizes[0] else options[0][0]
        return {"mode": mode, "singleton_bytes_estimate": sizes[0], "mixed_bytes_estimate": sizes[1],
                "singleton_seconds": seconds[0], "mixed_seconds": seconds[1]}
