// cbq_fixed_wd.cu -- k_linear_fixed instantiations for bit widths 14 15 16.
#include "cbq_fixed_launch.cuh"
namespace cbq {
CBQ_INSTANTIATE_FIXED(14)
CBQ_INSTANTIATE_FIXED(15)
CBQ_INSTANTIATE_FIXED(16)
}  // namespace cbq
