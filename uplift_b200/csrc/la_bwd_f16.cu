// Local Attender backward kernels stored as __half: every K, unit and
// vector-width variant (compiled on its own so the three storage types
// build in parallel).
#include "la_bwd.cuh"

namespace ula {
namespace bwd {

template int launch_k<__half>(const Args&, const Plan&, int, bool, bool, cudaStream_t);

}  // namespace bwd
}  // namespace ula
