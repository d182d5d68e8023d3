// Kernel table for one GGUF type (split per type so the builds run in parallel).
#include "mmvq.cuh"
ANVIL_MMVQ_TABLE_RT(mmvq_kernel_iq2xxs, kTypeIQ2_XXS)
