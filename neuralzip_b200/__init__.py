"""NeuralZip decompression path for NVIDIA B200 (sm_100a).

Same entry points as the reference package (neuralzip/__init__.py:1-16):

    from neuralzip_b200 import neuralzip
    neuralzip()                       # transparent Transformers integration
    setup = neuralzip.setup(model)    # offline clustering + codebooks

Weights stay Huffman-coded in HBM and are rebuilt bit-exactly by the tile
decode kernel of libnzb200.so right before each block runs.
"""


class _NeuralZip:
    def __call__(self, setup=None, *, device=None):
        from neuralzip_b200.gpu.pretrained import enable

        return enable(setup, device=device)

    def setup(self, model, **options):
        from neuralzip_b200.setup import NeuralZipSetup

        return NeuralZipSetup(**options).build(model)


neuralzip = _NeuralZip()

__all__ = ["neuralzip"]
