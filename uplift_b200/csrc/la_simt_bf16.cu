// CUDA-core Local Attender kernels stored as __nv_bfloat16: every K, children-per-
// unit, vector-width and staged-guide variant (compiled on its own so the
// three storage types build in parallel).
#include "la_simt.cuh"

namespace ula {

KernelFn simt_kernel_bf16(int K, int cpt, bool vec, bool staged) { return pick_k<__nv_bfloat16>(K, cpt, vec, staged); }

}  // namespace ula
