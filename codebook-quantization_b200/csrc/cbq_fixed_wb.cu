// cbq_fixed_wb.cu -- k_linear_fixed instantiations for bit widths 7 8 9 10.
#include "cbq_fixed_launch.cuh"
namespace cbq {
CBQ_INSTANTIATE_FIXED(7)
CBQ_INSTANTIATE_FIXED(8)
CBQ_INSTANTIATE_FIXED(9)
CBQ_INSTANTIATE_FIXED(10)
}  // namespace cbq
