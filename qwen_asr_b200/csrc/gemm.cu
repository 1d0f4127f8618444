// GEMM dispatch. Every dense contraction of the encoder and the decoder prefill goes
// through gemm(); the implementation is selected here.
#include "common.h"
#include "kernels.h"

namespace qasr {

void gemm(const GemmArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return;
  gemm_simt(a, s);
}

}  // namespace qasr
