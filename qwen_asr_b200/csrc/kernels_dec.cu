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
                                const float* __restrict__ w, float eps, __nv_bfloat16* __restrict__ planes,
                                long long plane) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * d;
  float* yr = y + (size_t)blockIdx.x * d;
  float s = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
  float ss = block_sum(s, red);
  float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
  __nv_bfloat16* pr = planes ? planes + (size_t)blockIdx.x * d : nullptr;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
    yr[i] = v;
    if (pr) split3_bf16(v, pr[i], pr[i + plane], pr[i + 2 * plane]);
  }
}

void rms_norm_rows(const float* x, float* y, int rows, int d, const float* w, float eps, cudaStream_t s,
                   __nv_bfloat16* planes, long long plane) {
  if (rows > 0) rms_norm_kernel<<<rows, 256, 0, s>>>(x, y, d, w, eps, planes, plane);
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
                                                                 float* __restrict__ vc, int max_seq,
                                                                 const int* __restrict__ row_pos,
                                                                 const long long* __restrict__ row_kv) {
  __shared__ float sh[kHd];
  __shared__ float red[4];
  const int row = blockIdx.x, hh = blockIdx.y, d = threadIdx.x;
  const int ld = (n_heads + 2 * n_kv) * kHd;
  // packed rows of several sequences: each row's own position and KV slot offset
  const int pos = row_pos ? row_pos[row] : start + row;
  if (row_kv) {
    kc += row_kv[row];
    vc += row_kv[row];
  }
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
                                                 max_seq, nullptr, nullptr);
}

void prefill_qk_rope_kv_packed(float* qkv, int R, const int* row_pos, const long long* row_kv, int n_heads, int n_kv,
                               const float* qn, const float* kn, float eps, const float* rope_cos,
                               const float* rope_sin, float* kc, float* vc, int max_seq, cudaStream_t s) {
  if (R <= 0) return;
  dim3 grid(R, n_heads + n_kv);
  prefill_qk_rope_kv_kernel<<<grid, 128, 0, s>>>(qkv, 0, n_heads, n_kv, qn, kn, eps, rope_cos, rope_sin, kc, vc,
                                                 max_seq, row_pos, row_kv);
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

// ------------------------------------------------------------------ row argmax
// One block per row: each thread keeps its strided first maximum, then the block keeps the
// larger value, or the smaller index between equal values (the first maximum overall).
__global__ void rows_argmax_kernel(const float* __restrict__ x, int n, int* __restrict__ out) {
  const float* r = x + (size_t)blockIdx.x * n;
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;  // no element seen
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = r[i];
    if (bi == 0x7FFFFFFF || v > bv) {
      bv = v;
      bi = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7FFFFFFF;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7FFFFFFF ? 0 : bi;
  }
}

void rows_argmax(const float* x, int rows, int n, int* out, cudaStream_t s) {
  if (rows > 0 && n > 0) rows_argmax_kernel<<<rows, 256, 0, s>>>(x, n, out);
}

}  // namespace qasr
