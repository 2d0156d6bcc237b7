// gSpMM kernel instantiations for float (one translation unit per element type
// so the float and the other element type's kernels compile in parallel).
#include "spmm_launch.cuh"

namespace bgl {

template int launch_spmm_vj<float, 1, 1>(const SpmmArgs<float> &, int, int, cudaStream_t);
template int launch_spmm_vj<float, 4, 1>(const SpmmArgs<float> &, int, int, cudaStream_t);

}  // namespace bgl
