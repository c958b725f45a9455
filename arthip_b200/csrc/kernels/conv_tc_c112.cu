// Instantiations of the tcgen05 conv kernel for C = 112 input channels (every formulation
// and output variant), in a file of their own so the variants compile in parallel.
#include "conv_tc_kernel.cuh"

namespace ah {
namespace tck {

KernelFn kernel_c112(bool vert, int variant) { return pick<1, 1, 1>(vert, variant); }

}  // namespace tck
}  // namespace ah
