"""AxiomLM-B200: the quantized decode hot path of AxiomLM on sm_100a.

``ops``    -- the reference's ``_METAL_MOD`` op table on CUDA (libaxb.so)
``cache``  -- ``StaticKVCache`` in HBM
``model``  -- ``QuantizedDecoder`` (the CUDA-graph decode runner)
``medusa`` -- Medusa heads, tree compilation and speculative decoding (greedy on the device)
"""

__version__ = "0.1.0"


def load_library():
    """Load libaxb.so (raises ImportError if it has not been built)."""
    from . import _lib

    return _lib.load()
