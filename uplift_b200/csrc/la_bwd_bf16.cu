// Local Attender backward kernels stored as __nv_bfloat16: every K, unit and
// vector-width variant (compiled on its own so the three storage types
// build in parallel).
#include "la_bwd.cuh"

namespace ula {
namespace bwd {

template int launch_k<__nv_bfloat16>(const Args&, const Plan&, int, bool, bool, cudaStream_t);

}  // namespace bwd
}  // namespace ula
