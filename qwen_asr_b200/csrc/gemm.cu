// GEMM dispatch. Every dense contraction of the encoder and the decoder prefill goes
// through gemm(): the tcgen05 tensor-core kernel (gemm_tc.cu) for bf16 weight operands,
// the exact-FP32 SIMT kernel for f32 operands (mel tables). QASR_GEMM=simt forces the
// SIMT kernel (used by the parity tests as a second GPU reference).
#include <cstdlib>
#include <cstring>

#include "common.h"
#include "kernels.h"

namespace qasr {

static bool force_simt() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QASR_GEMM");
    v = (e && strcmp(e, "simt") == 0) ? 1 : 0;
  }
  return v == 1;
}

void gemm(const GemmArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return;
  if (!force_simt() && !a.b_is_f32 && gemm_tc(a, s)) return;
  gemm_simt(a, s);
}

}  // namespace qasr
