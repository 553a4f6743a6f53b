// CUDA-core Local Attender kernels stored as __half: every K, children-per-
// unit, vector-width and staged-guide variant (compiled on its own so the
// three storage types build in parallel).
#include "la_simt.cuh"

namespace ula {

KernelFn simt_kernel_f16(int K, int cpt, bool vec, bool staged) { return pick_k<__half>(K, cpt, vec, staged); }

}  // namespace ula
