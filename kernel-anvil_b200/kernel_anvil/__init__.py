"""kernel_anvil (B200 build): sm_100a MMVQ quantized GEMV kernels behind the
kernel-anvil surface -- smithy JSON configs, GGUF shape parsing and the
gguf-optimize / sweep / profile / merge-configs / autoforge CLI.

GPU ops live in ``kernel_anvil.mmvq`` (torch tensors over the C ABI of libanvil.so,
include/anvil.h).  Importing the package does not load the library.
"""
__version__ = "0.2.0"

from kernel_anvil.codegen import generate_config_header, generate_runtime_config  # noqa: F401,E402


def optimize(model, quant="Q8_0", verbose: bool = True, **launch):
    """Replace a model's nn.Linear layers with QuantLinear (see kernel_anvil.model.optimize);
    the reference's top-level kernel_anvil.optimize(model)."""
    from kernel_anvil.model import optimize as _optimize

    return _optimize(model, quant=quant, verbose=verbose, **launch)
