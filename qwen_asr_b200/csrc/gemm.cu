// GEMM dispatch. Every dense contraction of the encoder and the decoder prefill goes
// through gemm(): the tcgen05 tensor-core kernel (gemm_tc.cu) for bf16 weight operands,
// the exact-FP32 SIMT kernel for f32 operands (mel tables). QASR_GEMM=simt forces the
// SIMT kernel (used by the parity tests as a second GPU reference). A bf16-weight GEMM
// that the tensor-core kernel refuses is an error, not a silent slow path: it is counted
// (gemm_tc_fallbacks), recorded as the last error, and the engine fails the stage.
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

bool gemm_simt_forced() { return force_simt(); }

bool gemm(const GemmArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return true;
  if (a.b_is_f32 || force_simt()) {
    gemm_simt(a, s);
    return true;
  }
  if (gemm_tc(a, s)) return true;
  gemm_tc_note_fallback();
  set_error("tensor-core GEMM refused M=" + std::to_string(a.M) + " N=" + std::to_string(a.N) +
            " K=" + std::to_string(a.K) + " (computed by the SIMT kernel instead)");
  if (a.A) gemm_simt(a, s);
  return false;
}

}  // namespace qasr
