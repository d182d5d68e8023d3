// Kernel table for one GGUF type (split per type so the builds run in parallel).
#include "mmvq.cuh"
ANVIL_MMVQ_TABLE(mmvq_kernel_iq4xs, kTypeIQ4_XS)
