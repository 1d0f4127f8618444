// Mel front end and audio-encoder kernels (crates/qwen-asr/src/audio.rs:273-372,
// crates/qwen-asr/src/encoder.rs:186-358).
#include "common.h"
#include "dev_util.cuh"
#include "kernels.h"

namespace qasr {

// ------------------------------------------------------------------ mel front end
// Reflect-pad by 200 with zero fallback (audio.rs:280-291), frame t covers padded
// [t*160, t*160+400), multiplied by the periodic Hann window.
__global__ void mel_frames_kernel(const float* __restrict__ x, int n, int n_frames, const float* __restrict__ hann,
                                  float* __restrict__ frames) {
  long total = (long)n_frames * kNfft;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    int t = (int)(i / kNfft), k = (int)(i % kNfft);
    long p = (long)t * kHop + k;  // index into the padded signal
    float v;
    if (p < kNfft / 2) {
      long src = kNfft / 2 - p;
      v = src < n ? x[src] : 0.f;
    } else if (p < kNfft / 2 + n) {
      v = x[p - kNfft / 2];
    } else {
      long src = (long)n - 2 - (p - kNfft / 2 - n);
      v = src >= 0 ? x[src] : 0.f;
    }
    frames[i] = __fmul_rn(v, hann[k]);
  }
}

void mel_frames(const float* samples, int n, int n_frames, const float* hann, float* frames, cudaStream_t s) {
  long total = (long)n_frames * kNfft;
  int grid = (int)std::min<long>((total + 255) / 256, 148L * 16);
  mel_frames_kernel<<<grid, 256, 0, s>>>(samples, n, n_frames, hann, frames);
}

__global__ void mel_power_kernel(const float* __restrict__ spec, int ld_spec, int n_frames, float* __restrict__ pw,
                                 int ld_pow) {
  long total = (long)n_frames * ld_pow;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    int t = (int)(i / ld_pow), k = (int)(i % ld_pow);
    float v = 0.f;
    if (k < kNfreq) {
      float re = spec[(size_t)t * ld_spec + k], im = spec[(size_t)t * ld_spec + kNfreq + k];
      v = __fadd_rn(__fmul_rn(re, re), __fmul_rn(im, im));
    }
    pw[i] = v;
  }
}

void mel_power(const float* spec, int ld_spec, int n_frames, float* power, int ld_pow, cudaStream_t s) {
  long total = (long)n_frames * ld_pow;
  int grid = (int)std::min<long>((total + 255) / 256, 148L * 16);
  mel_power_kernel<<<grid, 256, 0, s>>>(spec, ld_spec, n_frames, power, ld_pow);
}

__global__ void mel_reset_kernel(int* g) { *g = float_to_ordered(-1e30f); }
void mel_reset_max(int* gmax, cudaStream_t s) { mel_reset_kernel<<<1, 1, 0, s>>>(gmax); }

__global__ void mel_normalize_kernel(float* m, long total, const int* gmax) {
  float lo = __fsub_rn(ordered_to_float(*gmax), 8.0f);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x)
    m[i] = __fdiv_rn(__fadd_rn(fmaxf(m[i], lo), 4.0f), 4.0f);
}

void mel_normalize(float* logmel, int n_frames, const int* gmax, cudaStream_t s) {
  long total = (long)n_frames * kMelBins;
  int grid = (int)std::min<long>((total + 255) / 256, 148L * 16);
  mel_normalize_kernel<<<grid, 256, 0, s>>>(logmel, total, gmax);
}

// ------------------------------------------------------------------ conv stem
// conv2d1: input image [128 mel bins (H)][w frames (W)], 1 channel.
__global__ void conv1_gelu_kernel(const float* __restrict__ mel, int n_frames, int f0, int cw, int w, int w1,
                                  const float* __restrict__ wt, const float* __restrict__ b,
                                  float* __restrict__ out, long total) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    int oc = (int)(i % kConvHidden);
    long r = i / kConvHidden;
    int ow = (int)(r % w1);
    r /= w1;
    int oh = (int)(r % 64);
    int c = (int)(r / 64);
    int frame0 = f0 + c * cw;
    float acc = 0.f;
#pragma unroll
    for (int ki = 0; ki < 3; ++ki) {
      int ih = 2 * oh + ki - 1;
#pragma unroll
      for (int kj = 0; kj < 3; ++kj) {
        int iw = 2 * ow + kj - 1;
        float v = (ih >= 0 && ih < kMelBins && iw >= 0 && iw < w) ? mel[(size_t)(frame0 + iw) * kMelBins + ih] : 0.f;
        acc = fmaf(wt[oc * 9 + ki * 3 + kj], v, acc);
      }
    }
    out[i] = gelu_tanh(__fadd_rn(acc, b[oc]));
  }
}

void conv1_gelu(const float* mel, int n_frames, int f0, int cw, int n_chunks, int w, const float* w1p,
                const float* b1, float* out, cudaStream_t s) {
  int w1 = (w + 2 - 3) / 2 + 1;
  long total = (long)n_chunks * 64 * w1 * kConvHidden;
  int grid = (int)std::min<long>((total + 255) / 256, 148L * 32);
  conv1_gelu_kernel<<<grid, 256, 0, s>>>(mel, n_frames, f0, cw, w, w1, w1p, b1, out, total);
}

// im2col over channels-last input; each thread moves 4 consecutive input channels. With
// `planes` the columns go straight to the tensor-core GEMM's three bf16 planes (no f32 copy).
__global__ void im2col_s2_kernel(const float* __restrict__ in, int H, int W, int Ho, int Wo, float* __restrict__ cols,
                                 bool col_major_rows, long total4, __nv_bfloat16* __restrict__ planes,
                                 long long plane) {
  const int K = 9 * kConvHidden;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total4; i += (long)gridDim.x * blockDim.x) {
    int k4 = (int)(i % (K / 4));
    long row = i / (K / 4);
    int ic = (k4 * 4) % kConvHidden, kk = (k4 * 4) / kConvHidden;
    int ki = kk / 3, kj = kk % 3;
    int per = Ho * Wo;
    int c = (int)(row / per), rr = (int)(row % per);
    int oh, ow;
    if (col_major_rows) {
      ow = rr / Ho;
      oh = rr % Ho;
    } else {
      oh = rr / Wo;
      ow = rr % Wo;
    }
    int ih = 2 * oh + ki - 1, iw = 2 * ow + kj - 1;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ih >= 0 && ih < H && iw >= 0 && iw < W)
      v = *reinterpret_cast<const float4*>(in + (((size_t)c * H + ih) * W + iw) * kConvHidden + ic);
    const size_t o = (size_t)row * K + kk * kConvHidden + ic;
    if (planes) {
      const float f[4] = {v.x, v.y, v.z, v.w};
      __nv_bfloat16 h[4], m[4], l[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) split3_bf16(f[j], h[j], m[j], l[j]);
      *reinterpret_cast<uint2*>(planes + o) = *reinterpret_cast<uint2*>(h);
      *reinterpret_cast<uint2*>(planes + plane + o) = *reinterpret_cast<uint2*>(m);
      *reinterpret_cast<uint2*>(planes + 2 * plane + o) = *reinterpret_cast<uint2*>(l);
    } else {
      *reinterpret_cast<float4*>(cols + o) = v;
    }
  }
}

void im2col_s2(const float* in, int n_chunks, int H, int W, float* cols, bool col_major_rows, cudaStream_t s,
               __nv_bfloat16* planes, long long plane) {
  int Ho = (H + 2 - 3) / 2 + 1, Wo = (W + 2 - 3) / 2 + 1;
  long total4 = (long)n_chunks * Ho * Wo * (9 * kConvHidden / 4);
  int grid = (int)std::min<long>((total4 + 255) / 256, 148L * 32);
  im2col_s2_kernel<<<grid, 256, 0, s>>>(in, H, W, Ho, Wo, cols, col_major_rows, total4, planes, plane);
}

__global__ void add_pe_kernel(float* x, long total, int d, int period, const float* pe) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    long r = i / d;
    int j = (int)(i % d);
    x[i] = __fadd_rn(x[i], pe[(r % period) * d + j]);
  }
}

void add_pe_rows(float* x, int rows, int d, int period, const float* pe, cudaStream_t s) {
  long total = (long)rows * d;
  int grid = (int)std::min<long>((total + 255) / 256, 148L * 16);
  add_pe_kernel<<<grid, 256, 0, s>>>(x, total, d, period, pe);
}

// ------------------------------------------------------------------ LayerNorm
// kernels/mod.rs:1160-1189: population variance, eps inside the sqrt.
__global__ void layer_norm_kernel(const float* __restrict__ x, float* __restrict__ y, int d,
                                  const float* __restrict__ w, const float* __restrict__ b, float eps,
                                  __nv_bfloat16* __restrict__ planes, long long plane) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * d;
  float* yr = y + (size_t)blockIdx.x * d;
  float s = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) s += xr[i];
  float mean = __fdiv_rn(block_sum(s, red), (float)d);
  float v = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float t = __fsub_rn(xr[i], mean);
    v = fmaf(t, t, v);
  }
  float var = __fdiv_rn(block_sum(v, red), (float)d);
  float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(var, eps)));
  __nv_bfloat16* pr = planes ? planes + (size_t)blockIdx.x * d : nullptr;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), w[i]), b[i]);
    yr[i] = v;
    if (pr) split3_bf16(v, pr[i], pr[i + plane], pr[i + 2 * plane]);
  }
}

void layer_norm_rows(const float* x, float* y, int rows, int d, const float* w, const float* b, float eps,
                     cudaStream_t s, __nv_bfloat16* planes, long long plane) {
  if (rows > 0) layer_norm_kernel<<<rows, 256, 0, s>>>(x, y, d, w, b, eps, planes, plane);
}

// ------------------------------------------------------------------ windowed attention
// One block per (window, head). K/V of the window staged in shared memory (rows padded to
// 65 floats against bank conflicts); one warp per query row; softmax over the window.
constexpr int kEncHd = 64;
__global__ void __launch_bounds__(256) window_attention_kernel(const float* __restrict__ qkv, float* __restrict__ out,
                                                               int d, const int* __restrict__ ws, float scale) {
  extern __shared__ float sm[];
  const int win = blockIdx.x, h = blockIdx.y;
  const int a = ws[win], b = ws[win + 1], L = b - a;
  float* Ks = sm;
  float* Vs = Ks + L * 65;
  float* Ps = Vs + L * 65;  // [8 warps][L]
  float* Qs = Ps + 8 * L;   // [8 warps][64]
  const int ld = 3 * d;
  for (int i = threadIdx.x; i < L * kEncHd; i += blockDim.x) {
    int r = i / kEncHd, c = i % kEncHd;
    const float* row = qkv + (size_t)(a + r) * ld + h * kEncHd + c;
    Ks[r * 65 + c] = row[d];
    Vs[r * 65 + c] = row[2 * d];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* P = Ps + warp * L;
  float* Q = Qs + warp * kEncHd;
  for (int qi = warp; qi < L; qi += 8) {
    const float* qrow = qkv + (size_t)(a + qi) * ld + h * kEncHd;
    Q[lane] = qrow[lane];
    Q[lane + 32] = qrow[lane + 32];
    __syncwarp();
    float mx = -3.0e38f;
    for (int j = lane; j < L; j += 32) {
      float acc = 0.f;
#pragma unroll 16
      for (int c = 0; c < kEncHd; ++c) acc = fmaf(Q[c], Ks[j * 65 + c], acc);
      float sc = __fmul_rn(acc, scale);
      P[j] = sc;
      mx = fmaxf(mx, sc);
    }
    mx = warp_max(mx);
    float sum = 0.f;
    for (int j = lane; j < L; j += 32) {
      float e = expf(__fsub_rn(P[j], mx));
      P[j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    float o0 = 0.f, o1 = 0.f;
    for (int j = 0; j < L; ++j) {
      float p = P[j];
      o0 = fmaf(p, Vs[j * 65 + lane], o0);
      o1 = fmaf(p, Vs[j * 65 + lane + 32], o1);
    }
    float inv = __fdiv_rn(1.0f, sum);
    float* orow = out + (size_t)(a + qi) * d + h * kEncHd;
    orow[lane] = __fmul_rn(o0, inv);
    orow[lane + 32] = __fmul_rn(o1, inv);
    __syncwarp();
  }
}

void enc_kernels_init() {
  cudaFuncSetAttribute(window_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

void window_attention(const float* qkv, float* out, int T, int d, int n_heads, const int* win_starts, int n_windows,
                      int max_win, float scale, cudaStream_t s) {
  (void)T;
  size_t smem = (size_t)(2 * max_win * 65 + 8 * max_win + 8 * kEncHd) * sizeof(float);
  dim3 grid(n_windows, n_heads);
  window_attention_kernel<<<grid, 256, smem, s>>>(qkv, out, d, win_starts, scale);
}

}  // namespace qasr
