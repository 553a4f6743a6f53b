// CUDA-core Local Attender kernels stored as float: every K, children-per-
// unit, vector-width and staged-guide variant (compiled on its own so the
// three storage types build in parallel).
#include "la_simt.cuh"

namespace ula {

KernelFn simt_kernel_f32(int K, int cpt, bool vec, bool staged) { return pick_k<float>(K, cpt, vec, staged); }

}  // namespace ula
