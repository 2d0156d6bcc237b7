// gSpMM kernel instantiations for double (one translation unit per element type
// so the double and the other element type's kernels compile in parallel).
#include "spmm_launch.cuh"

namespace bgl {

template int launch_spmm_vj<double, 1, 1>(const SpmmArgs<double> &, int, int, cudaStream_t);
template int launch_spmm_vj<double, 2, 1>(const SpmmArgs<double> &, int, int, cudaStream_t);

}  // namespace bgl
