"""turboembed_b200: a B200-native (sm_100a) CUDA backend for TurboEmbed's
encoder forward path, exported as the reference's `turbo_cuda_backend` table
(libturbo_b200.so). Python here only drives that C table for tests and
benchmarks; the compute is the library's CUDA kernels."""
from . import abi  # noqa: F401
