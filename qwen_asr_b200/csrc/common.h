// Shared definitions for the B200 Qwen3-ASR engine (host + device).
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace qasr {

// Constants of the model family (crates/qwen-asr/src/config.rs:3-24).
constexpr int kSampleRate = 16000;
constexpr int kMelBins = 128;
constexpr int kHop = 160;
constexpr int kNfft = 400;
constexpr int kNfreq = 201;
constexpr int kVocab = 151936;
constexpr int kConvHidden = 480;
constexpr int kTokImStart = 151644;
constexpr int kTokImEnd = 151645;
constexpr int kTokEndOfText = 151643;
constexpr int kTokAudioStart = 151669;
constexpr int kTokAudioEnd = 151670;
constexpr int kTokAsrText = 151704;
constexpr int kTokTimestamp = 151705;  // config.rs:20 (forced aligner)

// Verbosity shared by all engines (the reference keeps it global too, kernels/mod.rs:69).
extern int g_verbose;

void set_error(const std::string& msg);
std::string last_error();

#define QASR_LOG(level, ...)                                   \
  do {                                                         \
    if (::qasr::g_verbose >= (level)) fprintf(stderr, __VA_ARGS__); \
  } while (0)

// Records the failing CUDA call and returns `ret` from the enclosing function.
#define CUDA_OK(call, ret)                                                        \
  do {                                                                            \
    cudaError_t e__ = (call);                                                     \
    if (e__ != cudaSuccess) {                                                     \
      ::qasr::set_error(std::string(#call) + ": " + cudaGetErrorString(e__) +     \
                        " at " + __FILE__ + ":" + std::to_string(__LINE__));      \
      return ret;                                                                 \
    }                                                                             \
  } while (0)

inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

// Owning device allocation.
template <typename T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  bool alloc(size_t count) {
    if (count <= n && p) return true;
    release();
    if (count == 0) count = 1;
    if (cudaMalloc(&p, count * sizeof(T)) != cudaSuccess) {
      p = nullptr;
      set_error("cudaMalloc failed for " + std::to_string(count * sizeof(T)) + " bytes");
      return false;
    }
    n = count;
    return true;
  }
  bool upload(const T* host, size_t count, cudaStream_t s = 0) {
    if (!alloc(count)) return false;
    return cudaMemcpyAsync(p, host, count * sizeof(T), cudaMemcpyHostToDevice, s) == cudaSuccess;
  }
};

}  // namespace qasr
