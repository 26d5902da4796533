// ffn_stack_kernel instantiations: fast dequant path, one GPU.
#include "stack_launch.cuh"

namespace alv {
template int launch_stack_f<true, false>(alv_ctx*, const StackParams&, uint32_t,
                                                                      cudaStream_t);
}  // namespace alv
