"""Byte-lane layouts of the floating formats NeuralZip compresses.

Same contract as neuralzip/dtypes.py:8-83 (DTypeSpec and the three specs):
``reorder_bytes`` moves the sign below the exponent so that byte lane
``exponent_stream`` is the pure 8-bit exponent (bf16: lane 1, fp32: lane 3);
fp16 has no pure exponent lane and its GPU-coded lane is byte 1
(sign | exp5 | mant[9:8]).
"""

from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class DTypeSpec:
    name: str
    torch_dtype: torch.dtype
    numpy: np.dtype
    element_size: int
    bit_reorder: int
    mantissa_bits: int
    exponent_mask: int
    exponent_stream: int | None = None  # Only a byte stream of pure exponents.
    global_codebooks: tuple[tuple[int, str], ...] = ()

    @property
    def stream_ids(self):
        return range(self.element_size)

    @property
    def exponent_bits(self):
        return self.exponent_mask.bit_length()

    @property
    def gpu_stream(self):
        """Byte lane the GPU layout Huffman-codes (neuralzip/gpu/inference.py:299)."""
        return self.exponent_stream if self.exponent_stream is not None else self.element_size - 1

    def reorder_bytes(self, raw_bytes, *, restore=False):
        """Move the sign below the exponent, or undo it; layout 0 is identity."""
        if not self.bit_reorder:
            return raw_bytes
        unsigned = self.numpy.type
        exponent_bits = self.exponent_bits
        values = np.frombuffer(raw_bytes, dtype=self.numpy).copy()
        mantissa = values & unsigned((1 << self.mantissa_bits) - 1)
        if restore:
            sign = (values << unsigned(exponent_bits)) & unsigned(1 << (self.mantissa_bits + exponent_bits))
            exponent = (values >> unsigned(1)) & unsigned(self.exponent_mask << self.mantissa_bits)
        else:
            sign = (values >> unsigned(exponent_bits)) & unsigned(1 << self.mantissa_bits)
            exponent = (values << unsigned(1)) & unsigned(self.exponent_mask << (self.mantissa_bits + 1))
        return (sign | exponent | mantissa).astype(self.numpy, copy=False).tobytes()

    def extract_exponents(self, raw_bytes):
        """Extract exponent fields from original words, not from codec streams."""
        values = np.frombuffer(raw_bytes, dtype=self.numpy)
        return (values >> self.mantissa_bits) & self.exponent_mask


bfloat16 = DTypeSpec(
    name="bfloat16", torch_dtype=torch.bfloat16, numpy=np.dtype("<u2"), element_size=2,
    bit_reorder=1, mantissa_bits=7, exponent_mask=0xFF, exponent_stream=1,
)

float16 = DTypeSpec(
    name="float16", torch_dtype=torch.float16, numpy=np.dtype("<u2"), element_size=2,
    bit_reorder=0, mantissa_bits=10, exponent_mask=0x1F,
)

float32 = DTypeSpec(
    name="float32", torch_dtype=torch.float32, numpy=np.dtype("<u4"), element_size=4,
    bit_reorder=1, mantissa_bits=23, exponent_mask=0xFF, exponent_stream=3,
)

DTYPES = {spec.torch_dtype: spec for spec in (float16, bfloat16, float32)}
