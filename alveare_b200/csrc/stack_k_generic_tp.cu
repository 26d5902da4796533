// ffn_stack_kernel instantiations: generic dequant path, tensor-parallel ranks.
#include "stack_launch.cuh"

namespace alv {
template int launch_stack_f<false, true>(alv_ctx*, const StackParams&, uint32_t,
                                                                      cudaStream_t);
}  // namespace alv
