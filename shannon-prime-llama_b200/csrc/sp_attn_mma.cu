// sp_attn_mma.cu — tensor-core fused decode for the ship layout (placeholder
// until the kernel lands: reports the layout as unsupported so the generic
// kernel runs).
#include "sp_attn.cuh"

int sp_attn_mma_supported(const SpAttnArgs &) { return SP_ERR_UNSUPPORTED; }
int sp_attn_mma_launch(const SpAttnArgs &, cudaStream_t) { return SP_ERR_UNSUPPORTED; }
