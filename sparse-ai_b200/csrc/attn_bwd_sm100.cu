// Block-list attention backward on sm_100a (tcgen05).  Until the tensor-core backward lands,
// every shape is routed to the CUDA-core kernels of attn_simt.cu.
#include "attn_params.cuh"

namespace sa {

int launch_bwd_sm100(const AttnParams&, cudaStream_t, int) { return SA_EUNSUPPORTED; }

}  // namespace sa
