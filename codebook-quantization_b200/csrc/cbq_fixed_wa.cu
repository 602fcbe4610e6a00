// cbq_fixed_wa.cu -- k_linear_fixed instantiations for bit widths 1 2 3 4 5 6.
#include "cbq_fixed_launch.cuh"
namespace cbq {
CBQ_INSTANTIATE_FIXED(1)
CBQ_INSTANTIATE_FIXED(2)
CBQ_INSTANTIATE_FIXED(3)
CBQ_INSTANTIATE_FIXED(4)
CBQ_INSTANTIATE_FIXED(5)
CBQ_INSTANTIATE_FIXED(6)
}  // namespace cbq
