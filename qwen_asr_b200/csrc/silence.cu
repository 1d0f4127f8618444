// Silence compaction on the GPU (QwenCtx.skip_silence; audio.rs:375-479 compact_silence).
//
// The reference drops long pauses before transcription: per 10 ms window (160 samples) an
// RMS, an exponential smoothing s = 0.8 s + 0.2 rms, a threshold of 1.8 x the 25th
// percentile of the smoothed values clamped to [0.002, 0.025], voiced windows in runs of at
// least 5, each widened by 3 windows on both sides, and of every pause at most the first 60
// windows kept. Three launches:
//   1. window_rms_kernel   one thread per window; the window is staged through shared memory
//                          with coalesced loads and summed in sample order (x*x rounded, then
//                          added: the reference's loop), sqrt(e / len) correctly rounded;
//   2. silence_plan_kernel one CTA: the smoothing recurrence on one thread (f32 rounding after
//                          every operation, as the reference's sequential loop), the 25th
//                          percentile by a 4 x 8-bit radix select (non-negative floats order
//                          like their bit patterns), then the run filter, the widening, the
//                          pause rule (a window is kept when the last widened-voice window is
//                          at most 60 windows back) and the output offset of every kept window
//                          by block-wide scans;
//   3. silence_gather_kernel one thread per sample copies the kept windows.
// Every step after (1) is integer or order-free work, so the output equals the reference's
// sample for sample. When nothing is kept the first 0.5 s is returned, as the reference does.
#include "common.h"
#include "kernels.h"

namespace qasr {
namespace {

constexpr int kWin = 160;
constexpr int kRmsWindows = 64;  // windows per CTA of the RMS kernel (40 KB of samples)
constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kRmsWindows) window_rms_kernel(const float* __restrict__ x, long n, long n_win,
                                                                 float* __restrict__ rms) {
  __shared__ float s[kRmsWindows * (kWin + 1)];  // one padded row per window: conflict-free sums
  const long w0 = (long)blockIdx.x * kRmsWindows;
  const long a0 = w0 * kWin;
  const long avail = min((long)kRmsWindows * kWin, n - a0);
  for (long i = threadIdx.x; i < avail; i += blockDim.x) {
    const int w = (int)(i / kWin), j = (int)(i - (long)w * kWin);
    s[w * (kWin + 1) + j] = x[a0 + i];
  }
  __syncthreads();
  const long w = w0 + threadIdx.x;
  if (w >= n_win) return;
  const int len = (int)min((long)kWin, n - w * kWin);
  const float* row = s + threadIdx.x * (kWin + 1);
  float e = 0.f;
  for (int j = 0; j < len; ++j) e = __fadd_rn(e, __fmul_rn(row[j], row[j]));
  rms[w] = __fsqrt_rn(__fdiv_rn(e, (float)max(len, 1)));
}

template <typename T, typename Op>
__device__ T block_exclusive_scan(T v, T identity, Op op, T* sh /* [kPlanThreads / 32] */, T* total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  T inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc = op(inc, t);
  }
  if (lane == 31) sh[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    T wv = lane < kPlanThreads / 32 ? sh[lane] : identity;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T t = __shfl_up_sync(0xffffffffu, wv, o);
      if (lane >= o) wv = op(wv, t);
    }
    if (lane < kPlanThreads / 32) sh[lane] = wv;  // inclusive over warps
  }
  __syncthreads();
  const T before_warp = warp ? sh[warp - 1] : identity;
  T exc = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) exc = identity;
  const T out = op(before_warp, exc);
  if (total) *total = sh[kPlanThreads / 32 - 1];
  __syncthreads();
  return out;
}

struct MaxOp {
  __device__ long long operator()(long long a, long long b) const { return a > b ? a : b; }
};
struct SumOp {
  __device__ long long operator()(long long a, long long b) const { return a + b; }
};

__global__ void __launch_bounds__(kPlanThreads, 1)
    silence_plan_kernel(const float* __restrict__ rms, long n, long n_win, float* __restrict__ smooth,
                        unsigned char* __restrict__ voice, unsigned char* __restrict__ voice2,
                        unsigned char* __restrict__ pv, long long* __restrict__ offset, long long* count) {
  __shared__ unsigned int hist[256];
  __shared__ long long scan_sh[kPlanThreads / 32];
  __shared__ unsigned int sel_prefix, sel_mask, sel_k;
  __shared__ float thresh;
  const int tid = threadIdx.x;

  // smoothing recurrence (audio.rs: s = (1 - alpha) * s + alpha * rms, alpha = 0.2)
  if (tid == 0) {
    const float alpha = 0.2f, keep = 1.0f - 0.2f;
    float s = rms[0];
    for (long w = 0; w < n_win; ++w) {
      s = __fadd_rn(__fmul_rn(keep, s), __fmul_rn(alpha, rms[w]));
      smooth[w] = s;
    }
    sel_prefix = 0u;
    sel_mask = 0u;
    sel_k = (unsigned int)(long)((float)(n_win - 1) * 0.25f);  // p25 index of the sorted values
  }
  __syncthreads();

  // k-th smallest smoothed value: radix select over the bit patterns, 8 bits a pass
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kPlanThreads) hist[i] = 0u;
    __syncthreads();
    const unsigned int pre = sel_prefix, mask = sel_mask;
    for (long w = tid; w < n_win; w += kPlanThreads) {
      const unsigned int b = __float_as_uint(smooth[w]);
      if ((b & mask) == pre) atomicAdd(&hist[(b >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      unsigned int k = sel_k, bin = 0;
      while (hist[bin] <= k) {
        k -= hist[bin];
        ++bin;
      }
      sel_k = k;
      sel_prefix = pre | (bin << shift);
      sel_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  if (tid == 0) thresh = fminf(fmaxf(__fmul_rn(__uint_as_float(sel_prefix), 1.8f), 0.002f), 0.025f);
  __syncthreads();
  const float th = thresh;
  for (long w = tid; w < n_win; w += kPlanThreads) voice[w] = smooth[w] > th;
  __syncthreads();
  // voiced runs shorter than 5 windows are dropped
  for (long w = tid; w < n_win; w += kPlanThreads) {
    unsigned char v = voice[w];
    if (v) {
      int left = 0, right = 0;
      while (left < 4 && w - left - 1 >= 0 && voice[w - left - 1]) ++left;
      while (right < 4 && w + right + 1 < n_win && voice[w + right + 1]) ++right;
      v = left + right + 1 >= 5;
    }
    voice2[w] = v;
  }
  __syncthreads();
  // widened by 3 windows each side
  for (long w = tid; w < n_win; w += kPlanThreads) {
    unsigned char p = 0;
    for (long k = max(0L, w - 3); k <= min(n_win - 1, w + 3) && !p; ++k) p = voice2[k];
    pv[w] = p;
  }
  __syncthreads();
  // pause rule and output offsets, one contiguous run of windows per thread
  const long chunk = (n_win + kPlanThreads - 1) / kPlanThreads;
  const long c0 = min(n_win, tid * chunk), c1 = min(n_win, c0 + chunk);
  long long last = -1;
  for (long w = c0; w < c1; ++w)
    if (pv[w]) last = w;
  long long total = 0;
  const long long carry_last = block_exclusive_scan<long long>(last, -1LL, MaxOp(), scan_sh, nullptr);
  long long lp = carry_last, kept = 0;
  for (long w = c0; w < c1; ++w) {
    if (pv[w]) lp = w;
    if (pv[w] || w - lp <= 60) kept += min((long)kWin, n - w * kWin);
  }
  const long long base = block_exclusive_scan<long long>(kept, 0LL, SumOp(), scan_sh, &total);
  lp = carry_last;
  long long off = base;
  for (long w = c0; w < c1; ++w) {
    if (pv[w]) lp = w;
    if (pv[w] || w - lp <= 60) {
      offset[w] = off;
      off += min((long)kWin, n - w * kWin);
    } else {
      offset[w] = -1;
    }
  }
  if (tid == 0) {
    count[0] = total > 0 ? total : (long long)min(n, (long)kSampleRate / 2);
    count[1] = total == 0;
  }
}

// count = {kept samples, 1 when no window was kept (the first 0.5 s is copied instead)}
__global__ void silence_gather_kernel(const float* __restrict__ x, long n, const long long* __restrict__ offset,
                                      const long long* __restrict__ count, float* __restrict__ out) {
  const long long cnt = count[0];
  const bool none = count[1] != 0;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    if (none) {
      if (i < cnt) out[i] = x[i];
      continue;
    }
    const long w = i / kWin;
    const long long o = offset[w];
    if (o >= 0) out[o + (i - w * kWin)] = x[i];
  }
}

}  // namespace

size_t compact_silence_scratch(long n) {
  const long n_win = (n + kWin - 1) / kWin;
  // rms, smooth (f32); voice, voice2, pv (u8); offsets (i64)
  return (size_t)n_win * (4 + 4 + 3 + 8) + 256;
}

void compact_silence_device(const float* in, long n, float* out, void* scratch, long long* d_count,
                            cudaStream_t s) {
  const long n_win = (n + kWin - 1) / kWin;
  unsigned char* p = (unsigned char*)scratch;
  long long* offset = (long long*)p;
  float* rms = (float*)(offset + n_win);
  float* smooth = rms + n_win;
  unsigned char* voice = (unsigned char*)(smooth + n_win);
  unsigned char* voice2 = voice + n_win;
  unsigned char* pv = voice2 + n_win;
  window_rms_kernel<<<(unsigned)((n_win + kRmsWindows - 1) / kRmsWindows), kRmsWindows, 0, s>>>(in, n, n_win, rms);
  silence_plan_kernel<<<1, kPlanThreads, 0, s>>>(rms, n, n_win, smooth, voice, voice2, pv, offset, d_count);
  const long blocks = std::min<long>((n + 255) / 256, 148L * 16);
  silence_gather_kernel<<<(unsigned)blocks, 256, 0, s>>>(in, n, offset, d_count, out);
}

}  // namespace qasr
