"""B200-native backend for DotNetFoundryLLM's token loop.

The per-token forward pass over GGUF-quantized weights runs as hand-written
sm_100a kernels behind the C ABI in ``include/foundry_cuda.h``
(``_lib/libfoundry_cuda.so``).  The Python modules are the host-side mirror of
the reference's loader / forward-pass seam used by the tests and the
benchmark.
"""
__all__ = ["gguf", "ggufgen", "loader", "runtime", "build"]
