// Decoder kernels: prefill helpers and the single-token decode step
// (crates/qwen-asr/src/decoder.rs:455-645, kernels/mod.rs:838-1034, 1191-1240,
// 1480-1534, 1719-1893).
#include "common.h"
#include "dev_util.cuh"
#include "kernels.h"

namespace qasr {

constexpr int kHd = 128;  // decoder head_dim

// ------------------------------------------------------------------ RMSNorm rows
__global__ void rms_norm_kernel(const float* __restrict__ x, float* __restrict__ y, int d,
                                const float* __restrict__ w, float eps) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * d;
  float* yr = y + (size_t)blockIdx.x * d;
  float s = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
  float ss = block_sum(s, red);
  float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
  for (int i = threadIdx.x; i < d; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

void rms_norm_rows(const float* x, float* y, int rows, int d, const float* w, float eps, cudaStream_t s) {
  if (rows > 0) rms_norm_kernel<<<rows, 256, 0, s>>>(x, y, d, w, eps);
}

// Per-head RMSNorm (kernels/mod.rs:1214-1240) + NeoX RoPE (generic path :1780-1788) of a
// 128-vector held one element per thread; partner exchange through shared memory.
__device__ __forceinline__ float head_norm_rope(float v, const float* __restrict__ nw, float eps, float c, float sn,
                                                float* sh, float* red) {
  const int d = threadIdx.x;  // 0..127
  float ss = v * v;
  ss = warp_sum(ss);
  __syncthreads();
  if ((d & 31) == 0) red[d >> 5] = ss;
  __syncthreads();
  float tot = red[0] + red[1] + red[2] + red[3];
  float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)kHd), eps)));
  float nv = __fmul_rn(__fmul_rn(v, inv), nw[d]);
  sh[d] = nv;
  __syncthreads();
  float r;
  if (d < kHd / 2) {
    float x2 = sh[d + kHd / 2];
    r = __fadd_rn(__fmul_rn(nv, c), __fmul_rn(-x2, sn));
  } else {
    float x1 = sh[d - kHd / 2];
    r = __fadd_rn(__fmul_rn(nv, c), __fmul_rn(x1, sn));
  }
  __syncthreads();
  return r;
}

// grid (S, n_heads + n_kv), block 128.
__global__ void __launch_bounds__(128) prefill_qk_rope_kv_kernel(float* __restrict__ qkv, int start, int n_heads,
                                                                 int n_kv, const float* __restrict__ qn,
                                                                 const float* __restrict__ kn, float eps,
                                                                 const float* __restrict__ rc,
                                                                 const float* __restrict__ rs, float* __restrict__ kc,
                                                                 float* __restrict__ vc, int max_seq) {
  __shared__ float sh[kHd];
  __shared__ float red[4];
  const int row = blockIdx.x, hh = blockIdx.y, d = threadIdx.x;
  const int ld = (n_heads + 2 * n_kv) * kHd;
  const int pos = start + row;
  float c = rc[(size_t)pos * (kHd / 2) + (d & 63)], sn = rs[(size_t)pos * (kHd / 2) + (d & 63)];
  float* base = qkv + (size_t)row * ld;
  if (hh < n_heads) {
    float v = base[hh * kHd + d];
    base[hh * kHd + d] = head_norm_rope(v, qn, eps, c, sn, sh, red);
  } else {
    int kh = hh - n_heads;
    float v = base[(n_heads + kh) * kHd + d];
    float r = head_norm_rope(v, kn, eps, c, sn, sh, red);
    size_t off = ((size_t)kh * max_seq + pos) * kHd + d;
    kc[off] = r;
    vc[off] = base[(n_heads + n_kv + kh) * kHd + d];
  }
}

void prefill_qk_rope_kv(float* qkv, int S, int start, int n_heads, int n_kv, const float* qn, const float* kn,
                        float eps, const float* rope_cos, const float* rope_sin, float* kc, float* vc, int max_seq,
                        cudaStream_t s) {
  if (S <= 0) return;
  dim3 grid(S, n_heads + n_kv);
  prefill_qk_rope_kv_kernel<<<grid, 128, 0, s>>>(qkv, start, n_heads, n_kv, qn, kn, eps, rope_cos, rope_sin, kc, vc,
                                                 max_seq);
}

// ------------------------------------------------------------------ prefill attention
// grid (ceil(S/8), n_heads), block 256: one warp per query, key tiles of 32 staged in
// shared memory, online softmax.
constexpr int kPaTile = 32;
__global__ void __launch_bounds__(256) prefill_attention_kernel(const float* __restrict__ qkv, int S, int start,
                                                                int n_heads, int n_kv, const float* __restrict__ kc,
                                                                const float* __restrict__ vc, int max_seq, float scale,
                                                                float* __restrict__ out) {
  __shared__ float Ks[kPaTile][kHd + 1];
  __shared__ float Vs[kPaTile][kHd];
  __shared__ float Qs[8][kHd];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, kvh = h / (n_heads / n_kv);
  const int q0 = blockIdx.x * 8;
  const int qi = q0 + warp;
  const int ld = (n_heads + 2 * n_kv) * kHd;
  if (qi < S)
    for (int c = lane; c < kHd; c += 32) Qs[warp][c] = qkv[(size_t)qi * ld + h * kHd + c];
  const int my_last = start + qi;                            // last key this query may see
  const int blk_last = start + min(S - 1, q0 + 7);           // last key any query of the block sees
  float m = -3.0e38f, l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  const float* kb = kc + (size_t)kvh * max_seq * kHd;
  const float* vb = vc + (size_t)kvh * max_seq * kHd;
  for (int j0 = 0; j0 <= blk_last; j0 += kPaTile) {
    __syncthreads();
    for (int i = threadIdx.x; i < kPaTile * kHd / 4; i += 256) {
      int r = i / (kHd / 4), c4 = (i % (kHd / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (j0 + r <= blk_last) {
        kv = *reinterpret_cast<const float4*>(kb + (size_t)(j0 + r) * kHd + c4);
        vv = *reinterpret_cast<const float4*>(vb + (size_t)(j0 + r) * kHd + c4);
      }
      Ks[r][c4] = kv.x; Ks[r][c4 + 1] = kv.y; Ks[r][c4 + 2] = kv.z; Ks[r][c4 + 3] = kv.w;
      *reinterpret_cast<float4*>(&Vs[r][c4]) = vv;
    }
    __syncthreads();
    if (qi >= S) continue;
    int j = j0 + lane;
    float sc = -3.0e38f;
    if (j <= my_last) {
      float acc = 0.f;
#pragma unroll 16
      for (int c = 0; c < kHd; ++c) acc = fmaf(Qs[warp][c], Ks[lane][c], acc);
      sc = __fmul_rn(acc, scale);
    }
    float tmax = warp_max(sc);
    if (tmax <= -3.0e38f) continue;
    float mn = fmaxf(m, tmax);
    float corr = expf(__fsub_rn(m, mn));
    float p = j <= my_last ? expf(__fsub_rn(sc, mn)) : 0.f;
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int t = 0; t < 4; ++t) o[t] *= corr;
    for (int jj = 0; jj < kPaTile; ++jj) {
      float pj = __shfl_sync(0xffffffffu, p, jj);
      if (pj == 0.f) continue;
#pragma unroll
      for (int t = 0; t < 4; ++t) o[t] = fmaf(pj, Vs[jj][lane + 32 * t], o[t]);
    }
    m = mn;
  }
  if (qi < S) {
    float inv = __fdiv_rn(1.0f, l);
    float* orow = out + (size_t)qi * n_heads * kHd + h * kHd;
#pragma unroll
    for (int t = 0; t < 4; ++t) orow[lane + 32 * t] = __fmul_rn(o[t], inv);
  }
}

void prefill_attention(const float* qkv, int S, int start, int n_heads, int n_kv, const float* kc, const float* vc,
                       int max_seq, float scale, float* out, cudaStream_t s) {
  if (S <= 0) return;
  dim3 grid(ceil_div(S, 8), n_heads);
  prefill_attention_kernel<<<grid, 256, 0, s>>>(qkv, S, start, n_heads, n_kv, kc, vc, max_seq, scale, out);
}

// ------------------------------------------------------------------ prompt gather
__global__ void gather_embeds_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ embed,
                                     const float* __restrict__ enc, int d, float* __restrict__ out) {
  int r = blockIdx.x, id = ids[r];
  float* o = out + (size_t)r * d;
  if (id >= 0) {
    const uint16_t* e = reinterpret_cast<const uint16_t*>(embed) + (size_t)id * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) o[i] = bf16_bits_to_f32(e[i]);
  } else {
    const float* e = enc + (size_t)(-id - 1) * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) o[i] = e[i];
  }
}

void gather_embeds(const int* ids, int rows, const __nv_bfloat16* embed, const float* enc, int d, float* out,
                   cudaStream_t s) {
  if (rows > 0) gather_embeds_kernel<<<rows, 256, 0, s>>>(ids, embed, enc, d, out);
}

// ------------------------------------------------------------------ weight quantiser
// Per-row absmax int8 (kernels/mod.rs:1805-1829 with truncate=false; kernels/neon.rs:
// 637-694 with truncate=true): scale = absmax/127 (1 if absmax == 0),
// q = trunc|round(w * (127 / max(absmax, 1e-10))).
__global__ void quantize_rows_kernel(const __nv_bfloat16* __restrict__ w, int cols, bool truncate,
                                     int8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float red[32];
  const uint16_t* wr = reinterpret_cast<const uint16_t*>(w) + (size_t)blockIdx.x * cols;
  float mx = 0.f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) mx = fmaxf(mx, fabsf(bf16_bits_to_f32(wr[i])));
  mx = block_max(mx, red);
  float inv = __fdiv_rn(127.0f, fmaxf(mx, 1e-10f));
  if (threadIdx.x == 0) scale[blockIdx.x] = mx > 0.f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  int8_t* qr = q + (size_t)blockIdx.x * cols;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    float v = __fmul_rn(bf16_bits_to_f32(wr[i]), inv);
    float r = truncate ? truncf(v) : roundf(v);
    qr[i] = (int8_t)fminf(fmaxf(r, -127.f), 127.f);
  }
}

void quantize_rows_int8(const __nv_bfloat16* w, int rows, int cols, bool truncate, int8_t* q, float* scale,
                        cudaStream_t s) {
  if (rows > 0) quantize_rows_kernel<<<rows, 256, 0, s>>>(w, cols, truncate, q, scale);
}

// =====================================================================================
// Decode step
// =====================================================================================
__global__ void embed_kernel(const __nv_bfloat16* __restrict__ embed, int d, StepState* st, float* __restrict__ x) {
  int tok = st->cur_token;
  if (tok < 0) return;  // x already holds the input row (first step after prefill)
  const uint16_t* e = reinterpret_cast<const uint16_t*>(embed) + (size_t)tok * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) x[i] = bf16_bits_to_f32(e[i]);
}

enum MvEpi { MV_STORE = 0, MV_RESID = 1, MV_SWIGLU = 2, MV_ARGMAX = 3 };

struct MvArgs {
  const float* x;       // input vector [K]
  const float* norm_w;  // RMSNorm weight or null
  float eps;
  int K, N;
  const void* W;        // [N][K] int8 or bf16
  const float* ws;      // int8 row scales
  float* out;
  const float* resid;   // may alias out
  // argmax
  unsigned long long* am_part;
  int* am_ticket;
  StepState* st;
  int* tokens;
  const int* forced;
  float* logits;
};

// Packs (value, index) so that the max key is the max value, ties -> lowest index.
__device__ __forceinline__ unsigned long long am_key(float v, int idx) {
  unsigned int hv = (unsigned int)float_to_ordered(v) ^ 0x80000000u;
  return ((unsigned long long)hv << 32) | (unsigned int)(0xFFFFFFFFu - (unsigned int)idx);
}

// Prologue shared by all decode matvecs: stage x (optionally RMS-normalised) in shared
// memory and, for int8 weights, quantise it per vector (kernels/mod.rs:1795-1802).
template <bool INT8>
__device__ __forceinline__ float mv_prologue(const MvArgs& a, float* xs, int8_t* xq, float* red) {
  const int K = a.K;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(a.x + i);
    *reinterpret_cast<float4*>(xs + i) = v;
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  __syncthreads();  // xs is read below with a different thread mapping
  if (a.norm_w) {
    float tot = block_sum(ss, red);
    float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
    for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), a.norm_w[i]);
  }
  if (!INT8) {
    __syncthreads();
    return 1.0f;
  }
  float mx = 0.f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(xs[i]));
  mx = block_max(mx, red);
  float scale = mx > 0.f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  float inv = __fdiv_rn(127.0f, fmaxf(mx, 1e-10f));
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float r = roundf(__fmul_rn(xs[i], inv));
    xq[i] = (int8_t)fminf(fmaxf(r, -127.f), 127.f);
  }
  __syncthreads();
  return scale;
}

template <bool INT8, int EPI, int RPW>
__global__ void __launch_bounds__(256) matvec_kernel(MvArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[32];
  __shared__ unsigned long long am_warp[8];
  __shared__ int is_last;
  float* xs = reinterpret_cast<float*>(smem_raw);
  int8_t* xq = reinterpret_cast<int8_t*>(xs + a.K);
  const float xscale = mv_prologue<INT8>(a, xs, xq, red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K;
  unsigned long long best = 0ull;

  for (int rb = (blockIdx.x * 8 + warp) * RPW; rb < a.N; rb += gridDim.x * 8 * RPW) {
    float val[RPW];
    if (INT8) {
      int acc[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) acc[r] = 0;
      const int8_t* W = reinterpret_cast<const int8_t*>(a.W);
#pragma unroll 2
      for (int k0 = lane * 16; k0 < K; k0 += 512) {
        int4 xv = *reinterpret_cast<const int4*>(xq + k0);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          if (rb + r < a.N) {
            uint4 w = ld_stream(W + (size_t)(rb + r) * K + k0);
            acc[r] = __dp4a((int)w.x, xv.x, acc[r]);
            acc[r] = __dp4a((int)w.y, xv.y, acc[r]);
            acc[r] = __dp4a((int)w.z, xv.z, acc[r]);
            acc[r] = __dp4a((int)w.w, xv.w, acc[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        int s = warp_sum_i(acc[r]);
        val[r] = (rb + r < a.N) ? __fmul_rn(__fmul_rn((float)s, xscale), a.ws[rb + r]) : 0.f;
      }
    } else {
      float acc[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) acc[r] = 0.f;
      const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(a.W);
#pragma unroll 2
      for (int k0 = lane * 8; k0 < K; k0 += 256) {
        float4 x0 = *reinterpret_cast<const float4*>(xs + k0);
        float4 x1 = *reinterpret_cast<const float4*>(xs + k0 + 4);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          if (rb + r < a.N) {
            uint4 w = ld_stream(W + (size_t)(rb + r) * K + k0);
            float f[8];
            bf16x8_to_f32(w, f);
            acc[r] = fmaf(f[0], x0.x, acc[r]);
            acc[r] = fmaf(f[1], x0.y, acc[r]);
            acc[r] = fmaf(f[2], x0.z, acc[r]);
            acc[r] = fmaf(f[3], x0.w, acc[r]);
            acc[r] = fmaf(f[4], x1.x, acc[r]);
            acc[r] = fmaf(f[5], x1.y, acc[r]);
            acc[r] = fmaf(f[6], x1.z, acc[r]);
            acc[r] = fmaf(f[7], x1.w, acc[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RPW; ++r) val[r] = warp_sum(acc[r]);
    }
    if (EPI == MV_SWIGLU) {
      if (lane == 0)
#pragma unroll
        for (int r = 0; r + 1 < RPW; r += 2)
          if (rb + r + 1 < a.N) a.out[(rb + r) / 2] = silu_mul(val[r], val[r + 1]);
    } else if (EPI == MV_ARGMAX) {
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < RPW; ++r)
          if (rb + r < a.N) {
            if (a.logits) a.logits[rb + r] = val[r];
            unsigned long long k = am_key(val[r], rb + r);
            best = k > best ? k : best;
          }
    } else {
      if (lane < RPW) {
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < RPW; ++r)
          if (r == lane) v = val[r];
        int row = rb + lane;
        if (row < a.N) a.out[row] = EPI == MV_RESID ? __fadd_rn(v, a.resid[row]) : v;
      }
    }
  }

  if (EPI == MV_ARGMAX) {
    if (lane == 0) am_warp[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < 8; ++w) b = am_warp[w] > b ? am_warp[w] : b;
      a.am_part[blockIdx.x] = b;
      __threadfence();
      int t = atomicAdd(a.am_ticket, 1);
      is_last = (t == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      unsigned long long b = 0ull;
      for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
        unsigned long long v = *((volatile unsigned long long*)a.am_part + i);
        b = v > b ? v : b;
      }
      // block max of 64-bit keys
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
        b = t > b ? t : b;
      }
      if (lane == 0) am_warp[warp] = b;
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 0; w < 8; ++w) b = am_warp[w] > b ? am_warp[w] : b;
        int tok = (int)(0xFFFFFFFFu - (unsigned int)(b & 0xFFFFFFFFull));
        StepState* st = a.st;
        int step = st->step;
        a.tokens[step] = tok;
        st->cur_token = (st->forced_mode && a.forced) ? a.forced[step] : tok;
        st->step = step + 1;
        st->pos = st->pos + 1;
        *a.am_ticket = 0;
      }
    }
  }
}

template <bool INT8, int EPI, int RPW>
static void launch_mv(const MvArgs& a, int grid, cudaStream_t s) {
  size_t smem = (size_t)a.K * (INT8 ? 5 : 4) + 16;
  static int attr_done[16] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev < 16 && !attr_done[dev]) {
    cudaFuncSetAttribute(matvec_kernel<INT8, EPI, RPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    attr_done[dev] = 1;
  }
  matvec_kernel<INT8, EPI, RPW><<<grid, 256, smem, s>>>(a);
}

template <int EPI, int RPW>
static void mv(bool int8, const MvArgs& a, cudaStream_t s, int max_grid = 0) {
  int grid = ceil_div(a.N, 8 * RPW);
  if (max_grid > 0 && grid > max_grid) grid = max_grid;
  if (int8) launch_mv<true, EPI, RPW>(a, grid, s);
  else launch_mv<false, EPI, RPW>(a, grid, s);
}

// ------------------------------------------------------------------ decode attention
// grid (kv_heads, kSplits), block 128. Fuses q/k RMSNorm + RoPE + KV append with a
// split-K online-softmax attention over positions 0..pos; the last CTA of each kv head
// to finish merges the split partials (no spin-waits: arrival ticket only).
constexpr int kSplits = 16;
constexpr int kMaxG = 4;  // q heads per kv head supported

__global__ void __launch_bounds__(128) decode_attention_kernel(const float* __restrict__ qkv, int n_heads, int n_kv,
                                                               const float* __restrict__ qn,
                                                               const float* __restrict__ kn, float eps,
                                                               const float* __restrict__ rc,
                                                               const float* __restrict__ rs, float* __restrict__ kc,
                                                               float* __restrict__ vc, int max_seq, float scale,
                                                               StepState* st, float* __restrict__ part,
                                                               int* __restrict__ ticket, float* __restrict__ out) {
  __shared__ float sh[kHd];
  __shared__ float red[4];
  __shared__ float qs[kMaxG][kHd];
  __shared__ float ks[kHd], vs[kHd];
  __shared__ float wm[4][kMaxG], wl[4][kMaxG];
  __shared__ float wo[4][kMaxG][kHd];
  __shared__ int is_last;
  const int kvh = blockIdx.x, split = blockIdx.y, d = threadIdx.x;
  const int G = n_heads / n_kv;
  const int pos = st->pos;
  const float c = rc[(size_t)pos * (kHd / 2) + (d & 63)], sn = rs[(size_t)pos * (kHd / 2) + (d & 63)];
  for (int g = 0; g < G; ++g) qs[g][d] = head_norm_rope(qkv[(kvh * G + g) * kHd + d], qn, eps, c, sn, sh, red);
  ks[d] = head_norm_rope(qkv[(n_heads + kvh) * kHd + d], kn, eps, c, sn, sh, red);
  vs[d] = qkv[(n_heads + n_kv + kvh) * kHd + d];
  float* kb = kc + (size_t)kvh * max_seq * kHd;
  float* vb = vc + (size_t)kvh * max_seq * kHd;
  if (split == 0) {
    kb[(size_t)pos * kHd + d] = ks[d];
    vb[(size_t)pos * kHd + d] = vs[d];
  }
  __syncthreads();
  const int total = pos + 1;
  const int chunk = (total + kSplits - 1) / kSplits;
  const int j0 = split * chunk, j1 = min(total, j0 + chunk);
  const int warp = d >> 5, lane = d & 31;
  float m[kMaxG], l[kMaxG], o[kMaxG][4];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    m[g] = -3.0e38f;
    l[g] = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) o[g][t] = 0.f;
  }
  for (int j = j0 + warp; j < j1; j += 4) {
    float4 kv, vv;
    if (j == pos) {
      kv = *reinterpret_cast<const float4*>(&ks[lane * 4]);
      vv = *reinterpret_cast<const float4*>(&vs[lane * 4]);
    } else {
      kv = *reinterpret_cast<const float4*>(kb + (size_t)j * kHd + lane * 4);
      vv = *reinterpret_cast<const float4*>(vb + (size_t)j * kHd + lane * 4);
    }
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g >= G) break;
      float4 q = *reinterpret_cast<const float4*>(&qs[g][lane * 4]);
      float p = q.x * kv.x;
      p = fmaf(q.y, kv.y, p);
      p = fmaf(q.z, kv.z, p);
      p = fmaf(q.w, kv.w, p);
      float sc = __fmul_rn(warp_sum(p), scale);
      float mn = fmaxf(m[g], sc);
      float corr = expf(__fsub_rn(m[g], mn));
      float e = expf(__fsub_rn(sc, mn));
      l[g] = fmaf(l[g], corr, e);
      o[g][0] = fmaf(o[g][0], corr, e * vv.x);
      o[g][1] = fmaf(o[g][1], corr, e * vv.y);
      o[g][2] = fmaf(o[g][2], corr, e * vv.z);
      o[g][3] = fmaf(o[g][3], corr, e * vv.w);
      m[g] = mn;
    }
  }
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      wm[warp][g] = m[g];
      wl[warp][g] = l[g];
    }
    *reinterpret_cast<float4*>(&wo[warp][g][lane * 4]) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
  }
  __syncthreads();
  // CTA partial per head: {M, L, O[128]} at part[((h * kSplits) + split) * 130]
  for (int g = 0; g < G; ++g) {
    float M = fmaxf(fmaxf(wm[0][g], wm[1][g]), fmaxf(wm[2][g], wm[3][g]));
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 4; ++w) {
      float f = wl[w][g] > 0.f ? expf(__fsub_rn(wm[w][g], M)) : 0.f;
      L = fmaf(wl[w][g], f, L);
      O = fmaf(wo[w][g][d], f, O);
    }
    float* pp = part + ((size_t)(kvh * G + g) * kSplits + split) * (kHd + 2);
    pp[2 + d] = O;
    if (d == 0) {
      pp[0] = M;
      pp[1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (d == 0) is_last = (atomicAdd(&ticket[kvh], 1) == kSplits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int g = 0; g < G; ++g) {
    const volatile float* base = part + (size_t)(kvh * G + g) * kSplits * (kHd + 2);
    float M = -3.0e38f;
    for (int sp = 0; sp < kSplits; ++sp)
      if (base[sp * (kHd + 2) + 1] > 0.f) M = fmaxf(M, base[sp * (kHd + 2)]);
    float L = 0.f, O = 0.f;
    for (int sp = 0; sp < kSplits; ++sp) {
      float ls = base[sp * (kHd + 2) + 1];
      if (ls > 0.f) {
        float f = expf(__fsub_rn(base[sp * (kHd + 2)], M));
        L = fmaf(ls, f, L);
        O = fmaf(base[sp * (kHd + 2) + 2 + d], f, O);
      }
    }
    out[(kvh * G + g) * kHd + d] = __fdiv_rn(O, L);
  }
  if (d == 0) ticket[kvh] = 0;
}

void decode_step(const DecodeArgs& a, cudaStream_t s) {
  const int qd = a.q_heads * kHd, kvd = a.kv_heads * kHd;
  const float scale = 1.0f / sqrtf((float)kHd);
  embed_kernel<<<1, 256, 0, s>>>(a.embed, a.hidden, a.st, a.x);
  for (int l = 0; l < a.layers; ++l) {
    float* kc = a.k_cache + (size_t)l * a.kv_heads * a.max_seq * kHd;
    float* vc = a.v_cache + (size_t)l * a.kv_heads * a.max_seq * kHd;
    MvArgs m{};
    m.eps = a.eps;
    // QKV (input RMSNorm fused in the prologue)
    m.x = a.x; m.norm_w = a.n1[l]; m.K = a.hidden; m.N = qd + 2 * kvd;
    m.W = a.w_qkv[l]; m.ws = a.s_qkv[l]; m.out = a.qkv;
    mv<MV_STORE, 2>(a.int8, m, s);
    decode_attention_kernel<<<dim3(a.kv_heads, kSplits), 128, 0, s>>>(
        a.qkv, a.q_heads, a.kv_heads, a.qn[l], a.kn[l], a.eps, a.rope_cos, a.rope_sin, kc, vc, a.max_seq, scale,
        a.st, a.part, a.ticket, a.attn);
    // O projection + residual
    m = MvArgs{};
    m.eps = a.eps;
    m.x = a.attn; m.norm_w = nullptr; m.K = qd; m.N = a.hidden;
    m.W = a.w_o[l]; m.ws = a.s_o[l]; m.out = a.x; m.resid = a.x;
    mv<MV_RESID, 1>(a.int8, m, s);
    // gate/up (post-attention RMSNorm fused) + SwiGLU
    m = MvArgs{};
    m.eps = a.eps;
    m.x = a.x; m.norm_w = a.n2[l]; m.K = a.hidden; m.N = 2 * a.inter;
    m.W = a.w_gu[l]; m.ws = a.s_gu[l]; m.out = a.ffn;
    mv<MV_SWIGLU, 2>(a.int8, m, s);
    // down projection + residual
    m = MvArgs{};
    m.eps = a.eps;
    m.x = a.ffn; m.norm_w = nullptr; m.K = a.inter; m.N = a.hidden;
    m.W = a.w_down[l]; m.ws = a.s_down[l]; m.out = a.x; m.resid = a.x;
    mv<MV_RESID, 1>(a.int8, m, s);
  }
  MvArgs m{};
  m.eps = a.eps;
  m.x = a.x; m.norm_w = a.final_norm; m.K = a.hidden; m.N = a.vocab;
  m.W = a.lm_w; m.ws = a.lm_s;
  m.am_part = a.am_part; m.am_ticket = a.am_ticket; m.st = a.st; m.tokens = a.tokens; m.forced = a.forced;
  m.logits = a.logits;
  mv<MV_ARGMAX, 2>(a.int8, m, s, 148 * 4);
}

}  // namespace qasr
