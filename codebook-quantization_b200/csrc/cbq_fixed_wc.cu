// cbq_fixed_wc.cu -- k_linear_fixed instantiations for bit widths 11 12 13.
#include "cbq_fixed_launch.cuh"
namespace cbq {
CBQ_INSTANTIATE_FIXED(11)
CBQ_INSTANTIATE_FIXED(12)
CBQ_INSTANTIATE_FIXED(13)
}  // namespace cbq
