"""kernel_anvil (B200 build): sm_100a MMVQ quantized GEMV kernels behind the
kernel-anvil surface -- smithy JSON configs, GGUF shape parsing and the
gguf-optimize / sweep / profile / merge-configs / autoforge CLI.

GPU ops live in ``kernel_anvil.mmvq`` (torch tensors over the C ABI of libanvil.so,
include/anvil.h).  Importing the package does not load the library.
"""
__version__ = "0.2.0"

from kernel_anvil.codegen import generate_config_header, generate_runtime_config  # noqa: F401,E402
