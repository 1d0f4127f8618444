// Allocation-free variant of the mel front end.
//
// Some callers cannot allocate device memory while they run: code paths that already
// hold a fixed device-memory budget and treat any cudaMalloc as a failure, real-time
// audio threads that must not block on the allocator, or hosts that forbid new device
// allocations after start-up. For them qwen_asr_mel_noalloc() computes the same log-mel
// features as the normal path, but keeps its intermediate buffers (windowed frames,
// DFT spectrum, power spectrum, running maximum) in one file-scope device array that is
// part of the loaded library instead of in memory allocated per call.
#include <mutex>

#include "../../include/qwen_asr_ext.h"
#include "common.h"
#include "kernels.h"
#include "c_api_types.h"

namespace qasr {
namespace {

constexpr int kNoallocMaxFrames = QWEN_ASR_MEL_NOALLOC_MAX_FRAMES;  // 10 s of audio at 100 frames/s
constexpr int kSpecLd = 408, kPowLd = 208;
// frames [F][400] + spectrum [F][408] + power [F][208] floats, then the int max cell.
constexpr size_t kScratchFloats = (size_t)kNoallocMaxFrames * (kNfft + kSpecLd + kPowLd) + 64;

// Every GPU that loads the library holds this array (about 4 MB) until the process exits.
static __device__ __align__(256) float g_mel_scratch[kScratchFloats];

std::mutex g_setup_mu;
float* g_scratch_addr[64] = {nullptr};  // device address of g_mel_scratch, per device

// Resolves the array's device address on the current device (once per device). In host
// code `g_mel_scratch` names a host-side stand-in, so kernels must get this address. The
// cached address belongs to the device's primary context; a cudaDeviceReset destroys that
// context together with every engine's allocations, so engines (and this entry point) are
// only usable again in a process that reloads them - the cache is not refreshed.
float* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("mel_noalloc: no usable current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_mel_scratch);
    if (e != cudaSuccess) {
      set_error(std::string("mel_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
      return nullptr;
    }
    g_scratch_addr[dev] = (float*)p;
  }
  return g_scratch_addr[dev];
}

}  // namespace
}  // namespace qasr

extern "C" int32_t qwen_asr_mel_noalloc(QwenAsrEngine* e, const float* d_samples, int32_t n_samples, float* d_mel,
                                        int64_t mel_cap) {
  using namespace qasr;
  if (!e || !d_samples || !d_mel || n_samples <= 0) {
    set_error("mel_noalloc: null argument or empty input");
    return -1;
  }
  const int F = n_samples / kHop;  // same frame count as mel_spectrogram (audio.rs:293-294)
  if (F <= 0) {
    set_error("mel_noalloc: audio too short (" + std::to_string(n_samples) + " samples)");
    return -1;
  }
  if (F > kNoallocMaxFrames) {
    set_error("mel_noalloc: " + std::to_string(F) + " frames exceed the maximum of " +
              std::to_string(kNoallocMaxFrames) + " (" + std::to_string(kNoallocMaxFrames * kHop) + " samples)");
    return -1;
  }
  if ((int64_t)F * kMelBins > mel_cap) {
    set_error("mel_noalloc: output capacity too small");
    return -1;
  }
  Engine& eng = e->ctx.eng;
  // Runs on the engine's device and gives the caller back its current device on return.
  int prev = -1;
  cudaGetDevice(&prev);
  struct Restore {
    int dev;
    ~Restore() {
      if (dev >= 0) cudaSetDevice(dev);
    }
  } restore{prev};
  if (cudaSetDevice(eng.device()) != cudaSuccess) {
    set_error("mel_noalloc: cudaSetDevice failed");
    return -1;
  }
  float* base = scratch_for_current_device();
  if (!base) return -1;
  float* frames = base;
  float* spec = frames + (size_t)kNoallocMaxFrames * kNfft;
  float* power = spec + (size_t)kNoallocMaxFrames * kSpecLd;
  int* gmax = reinterpret_cast<int*>(power + (size_t)kNoallocMaxFrames * kPowLd);
  cudaStream_t s = eng.stream();

  mel_frames(d_samples, n_samples, F, eng.hann_table(), frames, s);
  GemmArgs g;
  g.M = F; g.N = kSpecLd; g.K = kNfft;
  g.A = frames; g.lda = kNfft; g.B = eng.dft_table(); g.b_is_f32 = true; g.ldb = kNfft;
  g.C = spec; g.ldc = kSpecLd;
  gemm_simt(g, s);
  mel_power(spec, kSpecLd, F, power, kPowLd, s);
  mel_reset_max(gmax, s);  // the cell keeps the previous call's value: restart it
  GemmArgs g2;
  g2.M = F; g2.N = kMelBins; g2.K = kPowLd;
  g2.A = power; g2.lda = kPowLd; g2.B = eng.mel_filter_table(); g2.b_is_f32 = true; g2.ldb = kPowLd;
  g2.C = d_mel; g2.ldc = kMelBins; g2.epi = EPI_LOG10_MAX; g2.gmax = gmax;
  gemm_simt(g2, s);
  mel_normalize(d_mel, F, gmax, s);
  cudaError_t err = cudaStreamSynchronize(s);
  if (err == cudaSuccess) err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error(std::string("mel_noalloc: ") + cudaGetErrorString(err));
    return -1;
  }
  return F;
}
