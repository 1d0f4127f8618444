// Single-token decode step (decoder_forward, crates/qwen-asr/src/decoder.rs:550-645) as a
// chain of programmatic-dependent launches. Every weight matvec CTA owns a contiguous
// slab of rows; its first tiles are pulled into shared memory with cp.async.bulk BEFORE
// griddepcontrol.wait, so the HBM stream of kernel i+1 overlaps the tail of kernel i.
//
// Numerics follow the reference's int8 path exactly: per-vector activation quantisation
// (kernels/mod.rs:1795-1802), exact int32 dot products (dp4a), then
// (float)sum * x_scale * w_scale[row] (+ residual) (kernels/neon.rs:716-800).
#include <cooperative_groups.h>
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <type_traits>

#include "bulk.cuh"
#include "common.h"
#include "dev_util.cuh"
#include "kernels.h"

namespace qasr {

constexpr int kHd = 128;
constexpr int kWarps = 16;  // decode matvec CTA: 512 threads
constexpr int kThreads = kWarps * 32;
constexpr int kSplits = 16;  // attention split-K CTAs per kv head
constexpr int kMaxG = 4;     // q heads per kv head
// qkv_attn_kernel threads: 8 warps with int8 weights; 4 with bf16, whose larger register
// and shared-memory footprint would otherwise keep the next kernel's CTAs (launched early
// under programmatic dependent launch) off the SM.
template <bool INT8>
constexpr int qa_threads() { return INT8 ? 256 : 128; }

enum MvEpi { MV_STORE = 0, MV_RESID = 1, MV_SWIGLU = 2, MV_ARGMAX = 3 };

constexpr int kMaxB = 8;  // sequences per batched decode launch

struct MvArgs {
  const float* x;              // input vectors [B][ldx]
  const __nv_bfloat16* embed;  // optional: take x_b from embed[st[b].cur_token] when >= 0
  float* x_out;                // the gathered embedding rows are written here by CTA 0
  const float* norm_w;         // fused RMSNorm weight or null
  float eps;
  int K, N;
  int B, ldx, ldo;             // batch, row stride of x (and x_out) and of out/resid
  const float* ws;             // int8 row scales
  float* out;                  // [B][ldo]
  const float* resid;          // [B][ldo], may alias out
  int rows_per_cta;            // multiple of block_rows
  int block_rows;              // R: 16, 32 or 64 weight rows per stage (R / 16 per warp)
  int nkc;                     // 512-byte column chunks per row
  int stages;
  int cps;                     // 512-byte chunks per ring stage (streaming kernel; divides nkc)
  unsigned long long* am_part; // [B][gridDim.x]
  int* am_ticket;
  StepState* st;               // [B]
  int* tokens;                 // [B][tokens_ld]
  int tokens_ld;
  const int* forced;
  float* logits;
  int* err;
  unsigned long long* tl;
  int* tl_count;
  int kind;
  int sum_threads;             // batched staging: threads owning sum-of-squares chunks (0: all)
  const void* staged;          // batched steps: the inputs as stage_kernel left them, or null
};

// Byte offset of the f32 per-sequence scales in an int8 staged buffer ([B][kpad] int8 first).
__host__ __device__ inline size_t staged_scale_off(int B, int kpad) { return ((size_t)B * kpad + 15) & ~(size_t)15; }

__device__ __forceinline__ unsigned long long am_key(float v, int idx) {
  unsigned int hv = (unsigned int)float_to_ordered(v) ^ 0x80000000u;
  return ((unsigned long long)hv << 32) | (unsigned int)(0xFFFFFFFFu - (unsigned int)idx);
}

struct Timeline {
  // Each kernel's CTA 0 reserves kRecords records at entry (one atomic, before its dependency
  // wait): {kind, t_entry, t_after_wait, t_exit}, then kRecords - 1 sub-phase records
  // {code, t, 0, 0} written with plain stores, so a stamp does not stall the CTA on a
  // returning atomic. code = 100 + 10 * kind + phase; unused records keep code kUnused.
  static constexpr int kRecords = 8;
  static constexpr unsigned long long kUnused = 0xFFFFFFFFull;
  unsigned long long* slot = nullptr;
  int nsub = 0;
  __device__ __forceinline__ void begin(unsigned long long* tl, int* cnt, int kind) {
    if (tl && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) {
      slot = tl + 4 * (size_t)atomicAdd(cnt, kRecords);
      slot[0] = (unsigned long long)kind;
      slot[1] = global_timer_ns();
      slot[2] = slot[3] = 0;
      for (int i = 1; i < kRecords; ++i) slot[4 * i] = kUnused;
    }
  }
  __device__ __forceinline__ void mark(int i) {
    if (slot) slot[i] = global_timer_ns();
  }
  __device__ __forceinline__ void sub(unsigned long long*, int*, int code) {
    if (slot && threadIdx.x == 0 && nsub < kRecords - 1) {
      unsigned long long* r = slot + 4 * (1 + nsub++);
      r[1] = global_timer_ns();
      r[2] = r[3] = 0;
      r[0] = (unsigned long long)code;
    }
  }
};

constexpr int kChunk = 512;  // bytes of a weight row per stage (32 lanes x 16 bytes)

__device__ __forceinline__ void tma_box(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Reduces v[0..RPW) over the warp; afterwards lane `row_lane` holds row r's sum.
template <int RPW, typename T>
__device__ __forceinline__ T warp_reduce_rows(const T* v, int lane) {
  if (RPW == 4) {
    T s0 = (lane & 16) ? v[2] : v[0], s1 = (lane & 16) ? v[3] : v[1];
    T t0 = (lane & 16) ? v[0] : v[2], t1 = (lane & 16) ? v[1] : v[3];
    s0 += __shfl_xor_sync(0xffffffffu, t0, 16);
    s1 += __shfl_xor_sync(0xffffffffu, t1, 16);
    T u = (lane & 8) ? s1 : s0, w = (lane & 8) ? s0 : s1;
    u += __shfl_xor_sync(0xffffffffu, w, 8);
    u += __shfl_xor_sync(0xffffffffu, u, 4);
    u += __shfl_xor_sync(0xffffffffu, u, 2);
    u += __shfl_xor_sync(0xffffffffu, u, 1);
    return u;
  } else if (RPW == 2) {
    T s = (lane & 16) ? v[1] : v[0], t = (lane & 16) ? v[0] : v[1];
    s += __shfl_xor_sync(0xffffffffu, t, 16);
    s += __shfl_xor_sync(0xffffffffu, s, 8);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    return s;
  } else {
    T s = v[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  }
}
// Reduces v[0..8) over the warp with the lane pairing of warp_sum (xor 16, 8, 4, 2, 1), so
// each result is bit-identical to warp_sum of that value; afterwards lane l holds value
// ((l >> 4) & 1) * 4 + ((l >> 3) & 1) * 2 + ((l >> 2) & 1).
template <typename T>
__device__ __forceinline__ T warp_reduce8(const T (&v)[kMaxB], int lane) {
  T s[4], t[2];
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T keep = h16 ? v[i + 4] : v[i], send = h16 ? v[i] : v[i + 4];
    s[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const T keep = h8 ? s[i + 2] : s[i], send = h8 ? s[i] : s[i + 2];
    t[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  T u = (h4 ? t[1] : t[0]) + __shfl_xor_sync(0xffffffffu, h4 ? t[0] : t[1], 4);
  u += __shfl_xor_sync(0xffffffffu, u, 2);
  u += __shfl_xor_sync(0xffffffffu, u, 1);
  return u;
}

// warp_reduce8 for four values: afterwards lane l holds value ((l >> 4) & 1) * 2 + ((l >> 3) & 1).
template <typename T>
__device__ __forceinline__ T warp_reduce4(const T (&v)[4], int lane) {
  T s[2];
  const bool h16 = lane & 16, h8 = lane & 8;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const T keep = h16 ? v[i + 2] : v[i], send = h16 ? v[i] : v[i + 2];
    s[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  T u = (h8 ? s[1] : s[0]) + __shfl_xor_sync(0xffffffffu, h8 ? s[0] : s[1], 8);
  u += __shfl_xor_sync(0xffffffffu, u, 4);
  u += __shfl_xor_sync(0xffffffffu, u, 2);
  u += __shfl_xor_sync(0xffffffffu, u, 1);
  return u;
}

template <int RPW>
__device__ __forceinline__ int lane_row(int lane) {
  return RPW == 4 ? ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1) : (RPW == 2 ? (lane >> 4) : 0);
}
template <int RPW>
__device__ __forceinline__ bool row_lane(int lane) {
  return RPW == 4 ? (lane & 7) == 0 : (RPW == 2 ? (lane & 15) == 0 : lane == 0);
}

// Single-sequence staging (B = 1; stage_all below gives the same bits for B > 1): stages
// sequence b's input vector in shared memory: gathered from the embedding (layer 0)
// or read from x, RMS-normalised when norm_w is set, and for int8 weights quantised per
// vector (kernels/mod.rs:1795-1802) into xq_b; returns the activation scale (1 for bf16).
template <bool INT8>
__device__ float stage_x(const MvArgs& a, int b, float* xs_b, int8_t* xq_b, const float* snw, float* red, int kpad) {
  const int tid = threadIdx.x, K = a.K;
  const uint16_t* erow = nullptr;
  if (a.embed) {
    int tok = a.st[b].cur_token;
    if (tok >= 0) erow = reinterpret_cast<const uint16_t*>(a.embed) + (size_t)tok * K;
  }
  const float* xsrc = a.x + (size_t)b * a.ldx;
  // Thread t holds elements 4t.., 4(t + kThreads).. in registers (at most kMaxV float4s):
  // the sum of squares accumulates in that order, every reduction has its own shared
  // buffer (one barrier each), and the vector is normalised and quantised in registers.
  constexpr int kMaxV = 3;  // K <= 3 * 4 * kThreads = 6144
  __shared__ float red_ss[kWarps], red_mx[kWarps];
  float4 v[kMaxV];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) {
    const int i = (tid + j * kThreads) * 4;
    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < K) {
      if (erow) {
        uint2 u = *reinterpret_cast<const uint2*>(erow + i);
        v[j] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                           __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
        if (blockIdx.x == 0) *reinterpret_cast<float4*>(a.x_out + (size_t)b * a.ldx + i) = v[j];
      } else {
        v[j] = *reinterpret_cast<const float4*>(xsrc + i);
      }
      ss = fmaf(v[j].x, v[j].x, ss);
      ss = fmaf(v[j].y, v[j].y, ss);
      ss = fmaf(v[j].z, v[j].z, ss);
      ss = fmaf(v[j].w, v[j].w, ss);
    }
  }
  const int warp = tid >> 5, lane = tid & 31;
  if (a.norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) red_ss[warp] = ss;
    __syncthreads();
    const float tot = warp_sum(lane < kWarps ? red_ss[lane] : 0.f);
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int i = (tid + j * kThreads) * 4;
      if (i < K) {
        v[j].x = __fmul_rn(__fmul_rn(v[j].x, inv), snw[i]);
        v[j].y = __fmul_rn(__fmul_rn(v[j].y, inv), snw[i + 1]);
        v[j].z = __fmul_rn(__fmul_rn(v[j].z, inv), snw[i + 2]);
        v[j].w = __fmul_rn(__fmul_rn(v[j].w, inv), snw[i + 3]);
      }
    }
  }
  for (int i = K + tid; i < kpad; i += kThreads) {  // padding past K multiplies zero weights
    xs_b[i] = 0.f;
    if (INT8) xq_b[i] = 0;
  }
  float xscale = 1.0f;
  if (INT8) {
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxV; ++j)
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
    mx = warp_max(mx);
    if (lane == 0) red_mx[warp] = mx;
    __syncthreads();
    mx = warp_max(lane < kWarps ? red_mx[lane] : 0.f);
    xscale = mx > 0.f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(127.0f, fmaxf(mx, 1e-10f));
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int i = (tid + j * kThreads) * 4;
      if (i < K) {
        const float f[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        char4 q;
        int8_t* qp = reinterpret_cast<int8_t*>(&q);
#pragma unroll
        for (int e = 0; e < 4; ++e) qp[e] = (int8_t)fminf(fmaxf(roundf(__fmul_rn(f[e], inv)), -127.f), 127.f);
        *reinterpret_cast<char4*>(xq_b + i) = q;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int i = (tid + j * kThreads) * 4;
      if (i < K) *reinterpret_cast<float4*>(xs_b + i) = v[j];
    }
  }
  (void)red;
  __syncthreads();
  return xscale;
}

// Batched bf16 staging keeps each 256-float chunk (one 512-byte weight chunk's inputs) so
// that lane L's 8 floats sit in two halves at L*4 and 128 + L*4: the two 16-byte loads of a
// warp each read 512 contiguous bytes (no bank conflicts). Float offset of the 4 elements
// 4c..4c+3 within a sequence's vector:
__device__ __forceinline__ int xperm4(int c) { return (c >> 6) * 256 + (c & 1) * 128 + ((c & 63) >> 1) * 4; }

// Stages the input vectors of all B (> 1) sequences at once: read from x (layer 0: gathered
// from the embedding, the rows also written to x_out by CTA 0), RMS-normalised when norm_w
// is set, and for int8 weights quantised per vector (kernels/mod.rs:1795-1802) into xq[b]
// with scale xscale[b] (bf16: the f32 vector goes to xs[b], xscale[b] = 1). Thread t < P
// owns the 4-element chunks c = t + P j of every sequence and accumulates them in order:
// with P = 512 that is the order of stage_x, with P = the fused QKV kernel's block size
// that kernel's order, so a batched step is bit-identical to single-sequence steps. Every load
// is unconditional (a row past B re-reads row B - 1 and is discarded) so the B loads are
// in flight together; the block-wide reductions are shared by all sequences. The int8
// path keeps chunk j = 0 in registers and needs no f32 staging buffer.
template <bool INT8>
__device__ void stage_all(const MvArgs& a, float* xs, int8_t* xq, const float* snw, float* red /* [kMaxB][kWarps] */,
                          float* sinv /* [2 * kMaxB] */, float* xscale, int kpad) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, K = a.K, B = a.B;
  const int nc = K >> 2, P = a.sum_threads ? a.sum_threads : kThreads;
  __shared__ int stok[kMaxB];
  if (a.embed) {
    if (tid < kMaxB) stok[tid] = tid < B ? a.st[tid].cur_token : -1;
    __syncthreads();
  }
  auto ldx = [&](int b, int c) -> float4 {
    const int bb = min(b, B - 1);
    if (a.embed) {  // layer 0 (the q/k/v projection only): the row of the current token
      const int tok = stok[bb];
      if (tok >= 0) {
        const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(a.embed) + (size_t)tok * K + 4 * c);
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                           __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
      }
    }
    return *reinterpret_cast<const float4*>(a.x + (size_t)bb * a.ldx + 4 * c);
  };
  auto normed = [&](float4 v, float inv, int c) -> float4 {
    const float4 w = *reinterpret_cast<const float4*>(snw + 4 * c);
    return make_float4(__fmul_rn(__fmul_rn(v.x, inv), w.x), __fmul_rn(__fmul_rn(v.y, inv), w.y),
                       __fmul_rn(__fmul_rn(v.z, inv), w.z), __fmul_rn(__fmul_rn(v.w, inv), w.w));
  };
  auto sumsq = [](float s, float4 v) {
    s = fmaf(v.x, v.x, s);
    s = fmaf(v.y, v.y, s);
    s = fmaf(v.z, v.z, s);
    return fmaf(v.w, v.w, s);
  };
  auto absmax = [](float m, float4 v) {
    return fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  };
  for (int i = K + tid; i < kpad; i += kThreads)  // padding past K multiplies zero weights
    for (int b = 0; b < B; ++b) {
      if (INT8) xq[(size_t)b * kpad + i] = 0;
      else xs[(size_t)b * kpad + xperm4(i >> 2) + (i & 3)] = 0.f;
    }
  const bool has0 = tid < min(P, nc);
  const int c0 = has0 ? tid : 0;
  float4 hold[kMaxB];
  float acc[kMaxB];  // sum of squares (norm) or max |x| (int8 without norm)
  // Sequences b >= B are skipped (break) in every per-sequence loop: a B = 1 launch does the
  // work of one sequence, with each sequence's summation order unchanged.
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) hold[b] = b < B ? ldx(b, c0) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    acc[b] = 0.f;
    if (b >= B) break;
    if (!has0) continue;
    if (!INT8 && b < B) *reinterpret_cast<float4*>(xs + (size_t)b * kpad + xperm4(c0)) = hold[b];
    if (a.embed && blockIdx.x == 0 && b < B && stok[b] >= 0)
      *reinterpret_cast<float4*>(a.x_out + (size_t)b * a.ldx + 4 * c0) = hold[b];
    acc[b] = a.norm_w ? sumsq(0.f, hold[b]) : absmax(0.f, hold[b]);
  }
  for (int c = tid + P; c < nc && tid < P; c += P) {  // chunks j >= 1
#pragma unroll
    for (int h = 0; h < kMaxB; h += 4) {  // four sequences' loads in flight (registers)
      if (h >= B) break;
      float4 t[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) t[i] = ldx(h + i, c);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int b = h + i;
        if (!INT8 && b < B) *reinterpret_cast<float4*>(xs + (size_t)b * kpad + xperm4(c)) = t[i];
        if (a.embed && blockIdx.x == 0 && b < B && stok[b] >= 0)
          *reinterpret_cast<float4*>(a.x_out + (size_t)b * a.ldx + 4 * c) = t[i];
        acc[b] = a.norm_w ? sumsq(acc[b], t[i]) : absmax(acc[b], t[i]);
      }
    }
  }
  // per-sequence block reduction: warp butterflies, then warp b combines the 16 warp values
  auto reduce = [&](bool is_sum) {
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      if (b >= B) break;
      const float v = is_sum ? warp_sum(acc[b]) : warp_max(acc[b]);
      if (lane == 0 && b < B) red[b * kWarps + warp] = v;
    }
    __syncthreads();
    if (warp < B) {
      const float t = lane < kWarps ? red[warp * kWarps + lane] : (is_sum ? 0.f : -3.0e38f);
      const float r = is_sum ? warp_sum(t) : warp_max(t);
      if (lane == 0) {
        if (is_sum) {
          sinv[warp] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(r, (float)K), a.eps)));  // norm
        } else {
          xscale[warp] = r > 0.f ? __fdiv_rn(r, 127.0f) : 1.0f;
          sinv[kMaxB + warp] = __fdiv_rn(127.0f, fmaxf(r, 1e-10f));  // quantisation
        }
      }
    }
    __syncthreads();
  };
  if (!INT8 && tid < B) xscale[tid] = 1.0f;
  if (a.norm_w) {
    reduce(true);
    if (INT8) {
#pragma unroll
      for (int b = 0; b < kMaxB; ++b) {
        if (b >= B) break;
        hold[b] = normed(hold[b], sinv[min(b, B - 1)], c0);
        acc[b] = has0 ? absmax(0.f, hold[b]) : 0.f;
      }
      for (int c = tid + P; c < nc && tid < P; c += P) {
#pragma unroll
        for (int h = 0; h < kMaxB; h += 4) {
          if (h >= B) break;
          float4 t[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) t[i] = ldx(h + i, c);
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[h + i] = absmax(acc[h + i], normed(t[i], sinv[min(h + i, B - 1)], c));
        }
      }
    } else {
      for (int i = tid; i < B * nc; i += kThreads) {
        const int b = i / nc, c = i - b * nc;
        float4* p = reinterpret_cast<float4*>(xs + (size_t)b * kpad + xperm4(c));
        *p = normed(*p, sinv[b], c);
      }
    }
  }
  if (INT8) {
    reduce(false);
    auto quant = [&](int b, int c, float4 v) {
      const float inv = sinv[kMaxB + b];
      auto q = [&](float f) -> int {
        const float r = roundf(__fmul_rn(f, inv));
        return (int)fminf(fmaxf(r, -127.f), 127.f) & 0xFF;
      };
      *reinterpret_cast<int*>(xq + (size_t)b * kpad + 4 * c) = q(v.x) | (q(v.y) << 8) | (q(v.z) << 16) | (q(v.w) << 24);
    };
#pragma unroll
    for (int b = 0; b < kMaxB; ++b)
      if (has0 && b < B) quant(b, c0, hold[b]);
    for (int c = tid + P; c < nc && tid < P; c += P) {
#pragma unroll
      for (int h = 0; h < kMaxB; h += 4) {
        if (h >= B) break;
        float4 t[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) t[i] = ldx(h + i, c);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (h + i < B) quant(h + i, c, a.norm_w ? normed(t[i], sinv[h + i], c) : t[i]);
      }
    }
  }
  __syncthreads();
}

// The batched matvecs' inputs as stage_kernel computed them once for the whole grid: int8
// vectors [B][kpad] and their scales, or normalised f32 vectors [B][kpad] in the permuted
// layout the dot loops read. Copied verbatim, so the kernel sees the bits stage_all gives.
template <bool INT8>
__device__ void load_staged(const MvArgs& a, float* xs, int8_t* xq, float* xscale, int kpad) {
  const int tid = threadIdx.x, B = a.B;
  if (INT8) {
    const int4* src = reinterpret_cast<const int4*>(a.staged);
    int4* dst = reinterpret_cast<int4*>(xq);
    for (int i = tid; i < B * kpad / 16; i += kThreads) dst[i] = __ldcg(src + i);
    const float* sc = reinterpret_cast<const float*>(reinterpret_cast<const unsigned char*>(a.staged) +
                                                     staged_scale_off(B, kpad));
    if (tid < B) xscale[tid] = __ldcg(sc + tid);
  } else {
    const float4* src = reinterpret_cast<const float4*>(a.staged);
    float4* dst = reinterpret_cast<float4*>(xs);
    for (int i = tid; i < B * kpad / 4; i += kThreads) dst[i] = __ldcg(src + i);
    if (tid < B) xscale[tid] = 1.0f;
  }
  __syncthreads();
}

// Batched steps: the input staging (RMSNorm, int8 quantisation, embedding gather) of the
// next matvec, done once by one CTA with stage_all's threads and order and written to
// a.staged, instead of by every CTA of the matvec (each of which would otherwise read all B
// input vectors from L2, two or three times).
template <bool INT8>
__global__ void __launch_bounds__(kThreads, 1) stage_kernel(MvArgs a) {
  // one CTA per sequence (blockIdx.y): each sequence's staging is independent (its own block
  // reductions), so a one-sequence stage_all gives the bits the all-sequence one does
  Timeline tline;
  tline.begin(a.tl, a.tl_count, a.kind);
  extern __shared__ unsigned char sm_raw[];
  __shared__ float red[kMaxB * kWarps];
  __shared__ float sinv[2 * kMaxB];
  __shared__ float xscale[kMaxB];
  unsigned char* sm = (unsigned char*)(((uintptr_t)sm_raw + 15) & ~(uintptr_t)15);
  const int tid = threadIdx.x, b = blockIdx.y, K = a.K;
  const int kpad = a.nkc * kChunk / (INT8 ? 1 : 2);
  MvArgs s1 = a;
  s1.B = 1;
  s1.x = a.x + (size_t)b * a.ldx;
  if (a.x_out) s1.x_out = a.x_out + (size_t)b * a.ldx;
  s1.st = a.st + b;
  float* xs = reinterpret_cast<float*>(sm);                      // bf16: [kpad]
  int8_t* xq = reinterpret_cast<int8_t*>(xs + (INT8 ? 0 : kpad));  // int8: [kpad]
  float* snw = reinterpret_cast<float*>(xq + (INT8 ? kpad : 0));
  if (a.norm_w)
    for (int i = tid; i < K; i += kThreads) snw[i] = a.norm_w[i];
  pdl_launch_dependents();
  pdl_wait();
  tline.mark(2);
  stage_all<INT8>(s1, xs, xq, snw, red, sinv, xscale, kpad);
  unsigned char* out = reinterpret_cast<unsigned char*>(const_cast<void*>(a.staged));
  if (INT8) {
    const int4* src = reinterpret_cast<const int4*>(xq);
    int4* dst = reinterpret_cast<int4*>(out + (size_t)b * kpad);
    for (int i = tid; i < kpad / 16; i += kThreads) dst[i] = src[i];
    if (tid == 0) reinterpret_cast<float*>(out + staged_scale_off(a.B, kpad))[b] = xscale[0];
  } else {
    const float4* src = reinterpret_cast<const float4*>(xs);
    float4* dst = reinterpret_cast<float4*>(out) + (size_t)b * kpad / 4;
    for (int i = tid; i < kpad / 4; i += kThreads) dst[i] = src[i];
  }
  tline.mark(3);
}

// Greedy-token bookkeeping of sequence b after its argmax (decoder.rs:550-645 returns the
// token; transcribe.rs feeds it back as the next input).
__device__ __forceinline__ void commit_token(const MvArgs& a, int b, unsigned long long key) {
  const int tok = (int)(0xFFFFFFFFu - (unsigned int)(key & 0xFFFFFFFFull));
  StepState* st = a.st + b;
  const int step = st->step;
  a.tokens[(size_t)b * a.tokens_ld + step] = tok;
  st->cur_token = (st->forced_mode && a.forced) ? a.forced[step] : tok;
  st->step = step + 1;
  st->pos = st->pos + 1;
}

// Argmax finish shared by the matvec kernels: per-CTA best keys (best[b] in lane 0 of each
// warp after a warp reduction) -> am_part -> the last CTA to arrive reduces per sequence.
__device__ __forceinline__ void argmax_finish(const MvArgs& a, const unsigned long long (&best)[kMaxB],
                                              unsigned long long (*am_warp)[kMaxB], int* is_last) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    if (b >= a.B) break;
    unsigned long long v = best[b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long t2 = __shfl_xor_sync(0xffffffffu, v, o);
      v = t2 > v ? t2 : v;
    }
    if (lane == 0) am_warp[warp][b] = v;
  }
  __syncthreads();
  if (tid < a.B) {
    unsigned long long v = 0ull;
    for (int w = 0; w < kWarps; ++w) v = am_warp[w][tid] > v ? am_warp[w][tid] : v;
    a.am_part[(size_t)tid * gridDim.x + blockIdx.x] = v;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) *is_last = (atomicAdd(a.am_ticket, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!*is_last) return;
  __threadfence();
  for (int b = warp; b < a.B; b += kWarps) {
    unsigned long long v = 0ull;
    for (int i = lane; i < (int)gridDim.x; i += 32) {
      unsigned long long u = __ldcg(a.am_part + (size_t)b * gridDim.x + i);
      v = u > v ? u : v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long t2 = __shfl_xor_sync(0xffffffffu, v, o);
      v = t2 > v ? t2 : v;
    }
    if (lane == 0) commit_token(a, b, v);
  }
  __syncthreads();
  if (tid == 0) *a.am_ticket = 0;
}

// Decode matvec y_b = epi(W x_b) for B sequences sharing one weight stream. Each CTA owns
// rows_per_cta rows; the rows stream through a ring of shared-memory stages holding R rows
// x 512 bytes each (2-D TMA boxes; the first ones issued before the dependency wait).
// Every warp owns R/16 rows of a stage and accumulates them for every sequence across the
// row's 512-byte chunks, so all 16 warps work on every stage.
template <bool INT8, int EPI, int RPW, bool BATCH>
__global__ void __launch_bounds__(kThreads, 1) mv_kernel(const __grid_constant__ CUtensorMap wmap, MvArgs a) {
  Timeline tline;
  tline.begin(a.tl, a.tl_count, a.kind);
  extern __shared__ unsigned char sm_raw[];
  __shared__ float red_raw[BATCH ? kMaxB * kWarps : 32];
  __shared__ float sinv[BATCH ? 2 * kMaxB : 1];
  float* red = red_raw;
  __shared__ unsigned long long am_warp[kWarps][kMaxB];
  __shared__ float xscale[kMaxB];
  __shared__ int is_last;
  unsigned char* sm = (unsigned char*)(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K, R = a.block_rows, nkc = a.nkc, B = BATCH ? a.B : 1;
  const int cps = a.cps, nsc = nkc / cps;  // chunks per stage, stages per row block
  const int kpad = nkc * kChunk / (INT8 ? 1 : 2);  // padded vector length in elements
  const int stage_bytes = R * kChunk * cps;  // [chunk][R rows][512 B]
  unsigned char* wst = sm;
  float* xs = reinterpret_cast<float*>(sm + (size_t)a.stages * stage_bytes);  // int8: [kpad] (B = 1 staging); bf16: [B][kpad]
  int8_t* xq = reinterpret_cast<int8_t*>(xs + (INT8 ? kpad : B * kpad));    // int8: [B][kpad]
  uint64_t* full = reinterpret_cast<uint64_t*>(xq + (INT8 ? ((B * kpad + 15) & ~15) : 0));
  uint64_t* empty = full + a.stages;
  float* sws = reinterpret_cast<float*>(empty + a.stages);
  float* snw = sws + a.rows_per_cta;

  const int r0 = blockIdx.x * a.rows_per_cta;
  const int nrows = max(0, min(a.N, r0 + a.rows_per_cta) - r0);
  const int nblocks = (nrows + R - 1) / R;
  const int nt = nblocks * nsc;
  auto issue = [&](int t) {
    const int s = t % a.stages, kc0 = (t % nsc) * cps, row = r0 + (t / nsc) * R;
    mbar_expect_tx(&full[s], (uint32_t)stage_bytes);
    for (int c = 0; c < cps; ++c)
      tma_box(wst + (size_t)s * stage_bytes + (size_t)c * R * kChunk, &wmap, (kc0 + c) * (kChunk / 2), row, &full[s]);
  };
  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_mbar_init();
    for (int t = 0; t < min(a.stages, nt); ++t) issue(t);  // weights do not depend on x
  }
  if (INT8)
    for (int i = tid; i < nrows; i += kThreads) sws[i] = a.ws[r0 + i];
  if (a.norm_w)
    for (int i = tid; i < K; i += kThreads) snw[i] = a.norm_w[i];
  pdl_launch_dependents();
  pdl_wait();
  tline.mark(2);
  if constexpr (!BATCH) {
    const float sc = stage_x<INT8>(a, 0, xs, xq, snw, red, kpad);
    if (tid == 0) xscale[0] = sc;
    __syncthreads();
  } else if (a.staged) {
    load_staged<INT8>(a, xs, xq, xscale, kpad);
  } else {
    stage_all<INT8>(a, xs, xq, snw, red, sinv, xscale, kpad);
  }
  tline.sub(a.tl, a.tl_count, 103 + 10 * a.kind);

  unsigned long long best[kMaxB];
  int iacc[4][kMaxB];
  float facc[4][kMaxB];
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    best[b] = 0ull;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      iacc[r][b] = 0;
      facc[r][b] = 0.f;
    }
  }
  for (int t = 0; t < nt; ++t) {
    const int s = t % a.stages, blk = t / nsc;
    mbar_wait(&full[s], (uint32_t)(t / a.stages) & 1u, a.err, 1);
    if (t == a.stages - 1) tline.sub(a.tl, a.tl_count, 104 + 10 * a.kind);  // prefetched stages consumed
    // chunks in column order, so every lane accumulates a row exactly as with one chunk per stage
    for (int c = 0; c < cps; ++c) {
    const int kc = (t % nsc) * cps + c;
    const unsigned char* tw = wst + (size_t)s * stage_bytes + (size_t)c * R * kChunk + (size_t)(warp * RPW) * kChunk + lane * 16;
    if (INT8) {
      int4 w[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) w[r] = *reinterpret_cast<const int4*>(tw + r * kChunk);
#pragma unroll
      for (int b = 0; b < kMaxB; ++b) {
        if (b >= B) break;
        const int4 xv = *reinterpret_cast<const int4*>(xq + (size_t)b * kpad + kc * kChunk + lane * 16);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          iacc[r][b] = __dp4a(w[r].x, xv.x, iacc[r][b]);
          iacc[r][b] = __dp4a(w[r].y, xv.y, iacc[r][b]);
          iacc[r][b] = __dp4a(w[r].z, xv.z, iacc[r][b]);
          iacc[r][b] = __dp4a(w[r].w, xv.w, iacc[r][b]);
        }
      }
    } else {
      float f[RPW][8];
#pragma unroll
      for (int r = 0; r < RPW; ++r) bf16x8_to_f32(*reinterpret_cast<const uint4*>(tw + r * kChunk), f[r]);
#pragma unroll
      for (int b = 0; b < kMaxB; ++b) {
        if (b >= B) break;
        const float* xb = xs + (size_t)b * kpad + kc * (kChunk / 2) + lane * (BATCH ? 4 : 8);
        const float4 x0 = *reinterpret_cast<const float4*>(xb);
        const float4 x1 = *reinterpret_cast<const float4*>(xb + (BATCH ? 128 : 4));
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          float acc = facc[r][b];
          acc = fmaf(f[r][0], x0.x, acc); acc = fmaf(f[r][1], x0.y, acc);
          acc = fmaf(f[r][2], x0.z, acc); acc = fmaf(f[r][3], x0.w, acc);
          acc = fmaf(f[r][4], x1.x, acc); acc = fmaf(f[r][5], x1.y, acc);
          acc = fmaf(f[r][6], x1.z, acc); acc = fmaf(f[r][7], x1.w, acc);
          facc[r][b] = acc;
        }
      }
    }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (tid == 0 && t + a.stages < nt) {
      mbar_wait(&empty[s], (uint32_t)(t / a.stages) & 1u, a.err, 2);  // every warp is done with it
      issue(t + a.stages);
    }
    if (t % nsc == nsc - 1) {
      // row block finished: reduce, scale, epilogue for every sequence
      const int lr = blk * R + warp * RPW + lane_row<RPW>(lane);
      const int row = r0 + lr;
      const bool valid = row_lane<RPW>(lane) && lr < nrows;
#pragma unroll
      for (int b = 0; b < kMaxB; ++b) {
        if (b >= B) break;
        float v;
        if (INT8) {
          int col[4] = {iacc[0][b], RPW > 1 ? iacc[1][b] : 0, RPW > 2 ? iacc[2][b] : 0, RPW > 3 ? iacc[3][b] : 0};
          const int u = warp_reduce_rows<RPW>(col, lane);  // exact int32 sum
          v = lr < nrows ? __fmul_rn(__fmul_rn((float)u, xscale[b]), sws[lr]) : 0.f;
        } else {
          float col[4] = {facc[0][b], RPW > 1 ? facc[1][b] : 0.f, RPW > 2 ? facc[2][b] : 0.f,
                          RPW > 3 ? facc[3][b] : 0.f};
          v = warp_reduce_rows<RPW>(col, lane);
        }
        float* ob = a.out + (size_t)b * a.ldo;
        if (EPI == MV_SWIGLU) {
          const float up = __shfl_down_sync(0xffffffffu, v, RPW == 4 ? 8 : 16);  // the paired "up" row
          if (valid && (lane_row<RPW>(lane) & 1) == 0 && lr + 1 < nrows) ob[row / 2] = silu_mul(v, up);
        } else if (EPI == MV_ARGMAX) {
          if (valid) {
            if (a.logits) a.logits[(size_t)b * a.N + row] = v;
            unsigned long long k = am_key(v, row);
            best[b] = k > best[b] ? k : best[b];
          }
        } else if (EPI == MV_RESID) {
          if (valid) ob[row] = __fadd_rn(v, a.resid[(size_t)b * a.ldo + row]);
        } else {
          if (valid) ob[row] = v;
        }
      }
#pragma unroll
      for (int b = 0; b < kMaxB; ++b)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          iacc[r][b] = 0;
          facc[r][b] = 0.f;
        }
    }
  }
  if (EPI == MV_ARGMAX) argmax_finish(a, best, am_warp, &is_last);
  tline.mark(3);
}

// Small decode matvec (<= 48 rows per CTA: the o, gate/up and down projections): the CTA's
// whole weight slab arrives in ONE stage (one TMA box per 512-byte column chunk) issued
// before the dependency wait; the 16 warps split the (sequence, row, chunk) dot products,
// and each row's chunk partials are summed in a fixed order (deterministic for f32 too).
template <bool INT8, int EPI, bool BATCH>
__device__ __forceinline__ void mv_small_body(const CUtensorMap& wmap, const MvArgs& a) {
  Timeline tline;
  tline.begin(a.tl, a.tl_count, a.kind);
  extern __shared__ unsigned char sm_raw[];
  __shared__ float red_raw[BATCH ? kMaxB * kWarps : 32];
  __shared__ float sinv[BATCH ? 2 * kMaxB : 1];
  float* red = red_raw;
  __shared__ float xscale[kMaxB];
  __shared__ __align__(8) uint64_t bar;
  unsigned char* sm = (unsigned char*)(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K, nkc = a.nkc, R = a.rows_per_cta, B = a.B;
  const int kpad = nkc * kChunk / (INT8 ? 1 : 2);
  unsigned char* wst = sm;  // [kc][R rows][512 B]
  float* xs = reinterpret_cast<float*>(sm + (size_t)nkc * R * kChunk);  // int8: [kpad] (B = 1 staging); bf16: [B][kpad]
  int8_t* xq = reinterpret_cast<int8_t*>(xs + (INT8 ? kpad : B * kpad));
  float* sws = reinterpret_cast<float*>(xq + (INT8 ? ((B * kpad + 15) & ~15) : 0));
  float* snw = sws + ((R + 3) & ~3);  // 16-byte aligned: read as float4
  float* part = snw + K;  // [B][R][nkc] chunk partials (int32 bit patterns for int8)
  const int r0 = blockIdx.x * R;
  const int nrows = max(0, min(a.N, r0 + R) - r0);
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&bar, (uint32_t)(nkc * R * kChunk));
    for (int kc = 0; kc < nkc; ++kc) tma_box(wst + (size_t)kc * R * kChunk, &wmap, kc * (kChunk / 2), r0, &bar);
  }
  if (INT8)
    for (int i = tid; i < nrows; i += kThreads) sws[i] = a.ws[r0 + i];
  if (a.norm_w)
    for (int i = tid; i < K; i += kThreads) snw[i] = a.norm_w[i];
  pdl_launch_dependents();
  pdl_wait();
  tline.mark(2);
  if constexpr (!BATCH) {
    for (int b = 0; b < B; ++b) {
      const float sc = stage_x<INT8>(a, b, INT8 ? xs : xs + (size_t)b * kpad, xq + (size_t)b * kpad, snw, red, kpad);
      if (tid == 0) xscale[b] = sc;
    }
  } else if (a.staged) {
    load_staged<INT8>(a, xs, xq, xscale, kpad);
  } else {
    stage_all<INT8>(a, xs, xq, snw, red, sinv, xscale, kpad);
  }
  tline.sub(a.tl, a.tl_count, 100 + 10 * a.kind);
  mbar_wait(&bar, 0, a.err, 5);
  tline.sub(a.tl, a.tl_count, 101 + 10 * a.kind);
  if (BATCH) {
    // items of kRG rows x one 512-byte chunk: each sequence's input chunk is read once and
    // dotted with the kRG rows (rows past R repeat row R - 1 and are dropped; sequences past
    // B repeat sequence B - 1 and are dropped); every (row, sequence) dot product keeps the
    // single-sequence kernel's arithmetic
    if constexpr (INT8) {
    // int8: items of 2 rows x one chunk, all sequences at once (16-byte conflict-free input
    // loads make the input cheap; the 8-value reduction keeps the shuffle count low)
    constexpr int kRG = 2;
    const int sel = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    const int ngroups = (R + kRG - 1) / kRG;
    for (int it = warp; it < ngroups * nkc; it += kWarps) {
      const int rg = it / nkc, kc = it - rg * nkc, rb = rg * kRG;
      uint4 wv[kRG];
#pragma unroll
      for (int j = 0; j < kRG; ++j)
        wv[j] = *reinterpret_cast<const uint4*>(wst + ((size_t)kc * R + min(rb + j, R - 1)) * kChunk + lane * 16);
      int acc[kRG][kMaxB];
#pragma unroll
      for (int b = 0; b < kMaxB; ++b) {
        const int4 xv = *reinterpret_cast<const int4*>(xq + (size_t)min(b, B - 1) * kpad + kc * kChunk + lane * 16);
#pragma unroll
        for (int j = 0; j < kRG; ++j) {
          acc[j][b] = __dp4a((int)wv[j].x, xv.x, 0);
          acc[j][b] = __dp4a((int)wv[j].y, xv.y, acc[j][b]);
          acc[j][b] = __dp4a((int)wv[j].z, xv.z, acc[j][b]);
          acc[j][b] = __dp4a((int)wv[j].w, xv.w, acc[j][b]);
        }
      }
#pragma unroll
      for (int j = 0; j < kRG; ++j) {
        const int u = warp_reduce8(acc[j], lane);
        if ((lane & 3) == 0 && sel < B && rb + j < R) part[((size_t)sel * R + rb + j) * nkc + kc] = __int_as_float(u);
      }
    }
    } else {
    constexpr int kRG = 4;
    const int sel = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);  // warp_reduce4's value index
    const int ngroups = (R + kRG - 1) / kRG;
    for (int it = warp; it < ngroups * nkc; it += kWarps) {
      const int rg = it / nkc, kc = it - rg * nkc, rb = rg * kRG;
      uint4 wv[kRG];
#pragma unroll
      for (int j = 0; j < kRG; ++j)
        wv[j] = *reinterpret_cast<const uint4*>(wst + ((size_t)kc * R + min(rb + j, R - 1)) * kChunk + lane * 16);
      for (int bh = 0; bh < kMaxB / 4 && bh * 4 < B; ++bh) {  // sequences in groups of four
        float acc[kRG][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int b = min(bh * 4 + i, B - 1);
          const float* xb = xs + (size_t)b * kpad + kc * (kChunk / 2) + lane * 4;
          const float4 x0 = *reinterpret_cast<const float4*>(xb);
          const float4 x1 = *reinterpret_cast<const float4*>(xb + 128);
#pragma unroll
          for (int j = 0; j < kRG; ++j) {
            float f[8];
            bf16x8_to_f32(wv[j], f);
            float s = f[0] * x0.x;
            s = fmaf(f[1], x0.y, s); s = fmaf(f[2], x0.z, s); s = fmaf(f[3], x0.w, s);
            s = fmaf(f[4], x1.x, s); s = fmaf(f[5], x1.y, s); s = fmaf(f[6], x1.z, s);
            s = fmaf(f[7], x1.w, s);
            acc[j][i] = s;
          }
        }
#pragma unroll
        for (int j = 0; j < kRG; ++j) {
          const float u = warp_reduce4(acc[j], lane);
          const int b = bh * 4 + sel;
          if ((lane & 7) == 0 && b < B && rb + j < R) part[((size_t)b * R + rb + j) * nkc + kc] = u;
        }
      }
    }
  }
    }
  const int items = BATCH ? 0 : B * R * nkc;
  // bf16: four (sequence, row, chunk) items of a warp at a time, independent load / dot /
  // shuffle chains that overlap, each item computed exactly as on its own (int8 launches have
  // 2-6 items per warp, where the grouping measured slower).
  constexpr int kIlp = INT8 ? 1 : 4;
  for (int it0 = warp; it0 < items; it0 += kIlp * kWarps) {
    int its[kIlp];
#pragma unroll
    for (int u = 0; u < kIlp; ++u) its[u] = min(it0 + u * kWarps, items - 1);  // tail repeats the last item
    if (INT8) {
      int acc[kIlp];
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        const int it = its[u], b = it / (R * nkc), r = (it / nkc) % R, kc = it % nkc;
        const int4 xv = *reinterpret_cast<const int4*>(xq + (size_t)b * kpad + kc * kChunk + lane * 16);
        const int4 wv = *reinterpret_cast<const int4*>(wst + ((size_t)kc * R + r) * kChunk + lane * 16);
        acc[u] = __dp4a(wv.x, xv.x, 0);
        acc[u] = __dp4a(wv.y, xv.y, acc[u]);
        acc[u] = __dp4a(wv.z, xv.z, acc[u]);
        acc[u] = __dp4a(wv.w, xv.w, acc[u]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < kIlp; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);  // warp_sum_i
      if (lane == 0)
#pragma unroll
        for (int u = 0; u < kIlp; ++u)
          if (it0 + u * kWarps < items) part[its[u]] = __int_as_float(acc[u]);
    } else {
      float acc[kIlp];
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        const int it = its[u], b = it / (R * nkc), r = (it / nkc) % R, kc = it % nkc;
        const float* xb = xs + (size_t)b * kpad + kc * (kChunk / 2) + lane * 8;
        const float4 x0 = *reinterpret_cast<const float4*>(xb);
        const float4 x1 = *reinterpret_cast<const float4*>(xb + 4);
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(wst + ((size_t)kc * R + r) * kChunk + lane * 16), f);
        float v = f[0] * x0.x;
        v = fmaf(f[1], x0.y, v); v = fmaf(f[2], x0.z, v); v = fmaf(f[3], x0.w, v);
        v = fmaf(f[4], x1.x, v); v = fmaf(f[5], x1.y, v); v = fmaf(f[6], x1.z, v);
        v = fmaf(f[7], x1.w, v);
        acc[u] = v;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < kIlp; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);  // warp_sum
      if (lane == 0)
#pragma unroll
        for (int u = 0; u < kIlp; ++u)
          if (it0 + u * kWarps < items) part[its[u]] = acc[u];
    }
  }
  __syncthreads();
  tline.sub(a.tl, a.tl_count, 102 + 10 * a.kind);
  auto row_value = [&](int b, int r) -> float {
    const float* p = part + ((size_t)b * R + r) * nkc;
    if (INT8) {
      int s = 0;
      for (int kc = 0; kc < nkc; ++kc) s += __float_as_int(p[kc]);
      return __fmul_rn(__fmul_rn((float)s, xscale[b]), sws[r]);
    }
    float v = 0.f;
    for (int kc = 0; kc < nkc; ++kc) v += p[kc];
    return v;
  };
  if (EPI == MV_SWIGLU) {  // rows (2j, 2j+1) = (gate, up), r0 is even
    const int half = R / 2;
    for (int i = tid; i < B * half; i += kThreads) {
      const int b = i / half, j = i % half;
      if (2 * j + 1 < nrows) a.out[(size_t)b * a.ldo + (r0 >> 1) + j] = silu_mul(row_value(b, 2 * j), row_value(b, 2 * j + 1));
    }
  } else {
    for (int i = tid; i < B * R; i += kThreads) {
      const int b = i / R, r = i % R;
      if (r >= nrows) continue;
      const float v = row_value(b, r);
      const int row = r0 + r;
      if (EPI == MV_RESID) a.out[(size_t)b * a.ldo + row] = __fadd_rn(v, a.resid[(size_t)b * a.ldo + row]);
      else a.out[(size_t)b * a.ldo + row] = v;
    }
  }
  tline.mark(3);
}

// B = 1 instantiation, and the batched one (capped at 96 registers so a successor kernel's
// CTAs still fit beside it under programmatic dependent launch).
template <bool INT8, int EPI>
__global__ void __launch_bounds__(kThreads, 1) mv_small_kernel(const __grid_constant__ CUtensorMap wmap, MvArgs a) {
  mv_small_body<INT8, EPI, false>(wmap, a);
}
template <bool INT8, int EPI>
__global__ void __maxnreg__(96) mv_small_batch_kernel(const __grid_constant__ CUtensorMap wmap, MvArgs a) {
  mv_small_body<INT8, EPI, true>(wmap, a);
}

// ------------------------------------------------------------------ QKV + attention
// One cluster of kSplits CTAs per kv head, block 128 (one thread per head dimension).
// Phase 1 (QKV projection of this kv head's group, kernels/mod.rs:884-967): the group's
// (G+2)*128 rows (G q heads, k, v) are split evenly over the cluster; each CTA pulls its
// weight rows into shared memory with cp.async.bulk before the dependency wait, then
// RMS-normalises and (int8) quantises x and computes its rows. The cluster exchanges the
// q/k/v vectors through distributed shared memory.
// Phase 2: q/k RMSNorm (kernels/mod.rs:1214-1240) + NeoX RoPE + KV append at `pos`, then
// split-K online-softmax attention over positions 0..pos (kernels/mod.rs:1492-1534). K/V
// rows of earlier positions (written by earlier steps; StepState is constant within a
// step) are also pulled into shared memory before the wait. Split partials are merged
// through distributed shared memory (no global atomics).
// Split cluster barrier (arrive early, wait later). arrive.release / wait.acquire order the
// distributed-shared-memory stores before the barrier with the local loads after it.
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

struct QkvAttnArgs {
  const float* x;              // residual stream [K]
  const __nv_bfloat16* embed;  // layer 0: take x from embed[st->cur_token] when >= 0
  float* x_out;                // layer 0: gathered embedding row written by CTA (0, 0)
  const float* norm_w;         // input RMSNorm weight [K]
  float eps;
  int K;
  const void* W;               // [q + 2kv][K] int8 or bf16
  const float* ws;             // int8 row scales
  int n_heads, n_kv;
  const float* qn;
  const float* kn;
  const float* rc;
  const float* rs;
  float* kc;
  float* vc;
  int max_seq;
  float scale;
  int rows_per_cta;            // (G + 2) * 128 / kSplits
  int kv_rows;                 // K/V rows per CTA staged in shared memory
  StepState* st;
  float* out;                  // attention output [n_heads * 128]
  int ldx, ldo;                // per-sequence strides of x / x_out and out (blockIdx.z = sequence)
  size_t kv_slot_stride;       // floats between the KV caches of consecutive sequences
  int* err;
  unsigned long long* tl;
  int* tl_count;
  const float* qkv;            // attention-only variant: projected rows [B][ldq]
  int ldq;
};

template <bool INT8, bool PROJ, int MG>
__global__ void __launch_bounds__(PROJ ? qa_threads<INT8>() : 128, PROJ ? (INT8 ? 3 : 1) : 6)
qkv_attn_kernel(QkvAttnArgs a) {
  // The attention loop splits a CTA's positions over kVW virtual warps (the fused kernel's
  // warp count, which fixes the summation order); the attention-only variant runs them on
  // 4 warps, virtual warps w and w + 4 one after the other.
  constexpr int kQA = PROJ ? qa_threads<INT8>() : 128, kQAW = kQA / 32, kVW = qa_threads<INT8>() / 32;
  namespace cg = cooperative_groups;
  {  // sequence blockIdx.z of a batched step: its own residual row, state and KV slot
    const int b = blockIdx.z;
    a.x += (size_t)b * a.ldx;
    if (a.x_out) a.x_out += (size_t)b * a.ldx;
    a.out += (size_t)b * a.ldo;
    a.st += b;
    a.kc += (size_t)b * a.kv_slot_stride;
    a.vc += (size_t)b * a.kv_slot_stride;
    if (!PROJ) a.qkv += (size_t)b * a.ldq;
  }
  Timeline tline;
  tline.begin(a.tl, a.tl_count, 1);
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ __align__(8) uint64_t wbar, kvbar;
  __shared__ float vals[64];                          // this CTA's projected rows
  __shared__ __align__(16) float hv[MG + 2][kHd];  // normalised q heads, k, v of `pos`
  __shared__ float red[4][MG + 1];
  __shared__ float wm[kVW][MG], wl[kVW][MG];
  __shared__ __align__(16) float wo[kVW][MG][kHd];
  __shared__ float pm[MG], pl[MG];
  __shared__ __align__(16) float po[MG][kHd];
  // receive buffers written by the cluster's CTAs (distributed shared memory pushes)
  constexpr int kDimsPerCta = kHd / kSplits;
  __shared__ float allv[PROJ ? (MG + 2) * kHd : 1];                // the group's projected rows
  __shared__ float rcv_o[kSplits][MG][kDimsPerCta], rcv_m[kSplits][MG], rcv_l[kSplits][MG];
  cg::cluster_group cluster = cg::this_cluster();
  cluster_arrive_relaxed();  // "started": peers may push into this CTA once they wait on it
  const int kvh = blockIdx.x, rank = blockIdx.y, d = threadIdx.x;
  const int warp = d >> 5, lane = d & 31;
  const int G = a.n_heads / a.n_kv;
  const int K = a.K;
  const size_t row_bytes = (size_t)K * (INT8 ? 1 : 2);
  const int rpc = a.rows_per_cta;
  // shared-memory carve-up: weight rows | K rows | V rows | x f32 | x int8 | scales | norm w
  unsigned char* wsm = dsm;
  float* ksm = reinterpret_cast<float*>(dsm + (((size_t)rpc * row_bytes + 127) & ~(size_t)127));
  float* vsm = ksm + (size_t)a.kv_rows * kHd;
  float* xs = vsm + (size_t)a.kv_rows * kHd;
  int8_t* xq = reinterpret_cast<int8_t*>(xs + K);
  float* sws = reinterpret_cast<float*>(xq + ((K + 15) & ~15));
  float* snw = sws + 64;

  // ---- before the dependency wait
  const int pos = a.st->pos;
  const int total = pos + 1;
  const int chunk = (total + kSplits - 1) / kSplits;
  const int j0 = rank * chunk, j1 = min(total, j0 + chunk);
  const int npre = max(0, min(min(j1, pos) - j0, a.kv_rows));
  float* kb = a.kc + (size_t)kvh * a.max_seq * kHd;
  float* vb = a.vc + (size_t)kvh * a.max_seq * kHd;
  // Group row gi in [0, (G+2)*128) -> weight row (q heads, then k, then v of this kv head).
  auto wrow = [&](int gi) -> int {
    if (gi < G * kHd) return kvh * G * kHd + gi;
    if (gi < (G + 1) * kHd) return a.n_heads * kHd + kvh * kHd + (gi - G * kHd);
    return (a.n_heads + a.n_kv) * kHd + kvh * kHd + (gi - (G + 1) * kHd);
  };
  const int g0 = rank * rpc;
  if (d == 0) {
    mbar_init(&wbar, 1);
    mbar_init(&kvbar, 1);
    fence_mbar_init();
    if (PROJ) mbar_expect_tx(&wbar, (uint32_t)(rpc * row_bytes));
    // the CTA's rows form at most two runs (a q/k/v segment boundary may fall inside)
    int i = 0;
    while (PROJ && i < rpc) {
      int gi = g0 + i;
      int seg_end = (gi / kHd + 1) * kHd;
      int n = min(rpc - i, seg_end - gi);
      bulk_g2s(wsm + (size_t)i * row_bytes, reinterpret_cast<const unsigned char*>(a.W) + (size_t)wrow(gi) * row_bytes,
               (uint32_t)(n * row_bytes), &wbar);
      i += n;
    }
    if (npre > 0) {
      const uint32_t bytes = (uint32_t)(npre * kHd * sizeof(float));
      mbar_expect_tx(&kvbar, 2 * bytes);
      bulk_g2s(ksm, kb + (size_t)j0 * kHd, bytes, &kvbar);
      bulk_g2s(vsm, vb + (size_t)j0 * kHd, bytes, &kvbar);
    }
  }
  if (PROJ) {
    if (INT8 && d < rpc) sws[d] = a.ws[wrow(g0 + d)];
    for (int i = d; i < K; i += kQA) snw[i] = a.norm_w[i];
  }
  const int dd = d & (kHd - 1);  // head dimension of threads 0..127 (the rest help in loops)
  const float qn = a.qn[dd], kn = a.kn[dd];
  const float c = a.rc[(size_t)pos * (kHd / 2) + (dd & 63)], sn = a.rs[(size_t)pos * (kHd / 2) + (dd & 63)];
  pdl_launch_dependents();
  pdl_wait();
  tline.mark(2);

  if constexpr (PROJ) {
  // ---- phase 1: x -> RMSNorm -> (int8) -> this CTA's rows of q/k/v
  const uint16_t* erow = nullptr;
  if (a.embed) {
    int tok = a.st->cur_token;
    if (tok >= 0) erow = reinterpret_cast<const uint16_t*>(a.embed) + (size_t)tok * K;
  }
  // x, RMSNorm and the quantiser in registers: thread d holds elements 4d.., 4(d + kQA)..
  // (the sum of squares accumulates in that order), one barrier per block reduction
  constexpr int kMaxV = 4;  // K <= 4 * 4 * kQA
  __shared__ float red_ss[kQAW], red_mx[kQAW];
  float4 xv4[kMaxV];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) {
    const int i = (d + j * kQA) * 4;
    xv4[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < K) {
      if (erow) {
        uint2 b = *reinterpret_cast<const uint2*>(erow + i);
        xv4[j] = make_float4(__uint_as_float(b.x << 16), __uint_as_float(b.x & 0xFFFF0000u),
                             __uint_as_float(b.y << 16), __uint_as_float(b.y & 0xFFFF0000u));
        if (kvh == 0 && rank == 0) *reinterpret_cast<float4*>(a.x_out + i) = xv4[j];
      } else {
        xv4[j] = *reinterpret_cast<const float4*>(a.x + i);
      }
      ss = fmaf(xv4[j].x, xv4[j].x, ss);
      ss = fmaf(xv4[j].y, xv4[j].y, ss);
      ss = fmaf(xv4[j].z, xv4[j].z, ss);
      ss = fmaf(xv4[j].w, xv4[j].w, ss);
    }
  }
  {
    ss = warp_sum(ss);
    if (lane == 0) red_ss[warp] = ss;
    __syncthreads();
    const float tot = warp_sum(lane < kQAW ? red_ss[lane] : 0.f);
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int i = (d + j * kQA) * 4;
      if (i < K) {
        xv4[j].x = __fmul_rn(__fmul_rn(xv4[j].x, inv), snw[i]);
        xv4[j].y = __fmul_rn(__fmul_rn(xv4[j].y, inv), snw[i + 1]);
        xv4[j].z = __fmul_rn(__fmul_rn(xv4[j].z, inv), snw[i + 2]);
        xv4[j].w = __fmul_rn(__fmul_rn(xv4[j].w, inv), snw[i + 3]);
        *reinterpret_cast<float4*>(xs + i) = xv4[j];
      }
    }
  }
  float xscale = 1.0f;
  if (INT8) {
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxV; ++j)
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(xv4[j].x), fabsf(xv4[j].y)), fmaxf(fabsf(xv4[j].z), fabsf(xv4[j].w))));
    mx = warp_max(mx);
    if (lane == 0) red_mx[warp] = mx;
    __syncthreads();
    mx = warp_max(lane < kQAW ? red_mx[lane] : 0.f);
    xscale = mx > 0.f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(127.0f, fmaxf(mx, 1e-10f));
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int i = (d + j * kQA) * 4;
      if (i < K) {
        const float f[4] = {xv4[j].x, xv4[j].y, xv4[j].z, xv4[j].w};
        char4 q;
        int8_t* qp = reinterpret_cast<int8_t*>(&q);
#pragma unroll
        for (int e = 0; e < 4; ++e) qp[e] = (int8_t)fminf(fmaxf(roundf(__fmul_rn(f[e], inv)), -127.f), 127.f);
        *reinterpret_cast<char4*>(xq + i) = q;
      }
    }
  }
  __syncthreads();
  mbar_wait(&wbar, 0, a.err, 4);
  for (int rr = warp * 2; rr < rpc; rr += 2 * kQAW) {
    const bool two = rr + 1 < rpc;
    float v0, v1 = 0.f;
    if (INT8) {
      int acc0 = 0, acc1 = 0;
      const int8_t* w0 = reinterpret_cast<const int8_t*>(wsm) + (size_t)rr * K;
      const int8_t* w1 = w0 + K;
#pragma unroll 4
      for (int k0 = lane * 16; k0 < K; k0 += 512) {
        int4 xv = *reinterpret_cast<const int4*>(xq + k0);
        int4 wa = *reinterpret_cast<const int4*>(w0 + k0);
        acc0 = __dp4a(wa.x, xv.x, acc0);
        acc0 = __dp4a(wa.y, xv.y, acc0);
        acc0 = __dp4a(wa.z, xv.z, acc0);
        acc0 = __dp4a(wa.w, xv.w, acc0);
        if (two) {
          int4 wb = *reinterpret_cast<const int4*>(w1 + k0);
          acc1 = __dp4a(wb.x, xv.x, acc1);
          acc1 = __dp4a(wb.y, xv.y, acc1);
          acc1 = __dp4a(wb.z, xv.z, acc1);
          acc1 = __dp4a(wb.w, xv.w, acc1);
        }
      }
      acc0 = warp_sum_i(acc0);
      acc1 = warp_sum_i(acc1);
      v0 = __fmul_rn(__fmul_rn((float)acc0, xscale), sws[rr]);
      if (two) v1 = __fmul_rn(__fmul_rn((float)acc1, xscale), sws[rr + 1]);
    } else {
      float acc0 = 0.f, acc1 = 0.f;
      const uint16_t* w0 = reinterpret_cast<const uint16_t*>(wsm) + (size_t)rr * K;
      const uint16_t* w1 = w0 + K;
#pragma unroll 4
      for (int k0 = lane * 8; k0 < K; k0 += 256) {
        float4 x0 = *reinterpret_cast<const float4*>(xs + k0);
        float4 x1 = *reinterpret_cast<const float4*>(xs + k0 + 4);
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(w0 + k0), f);
        acc0 = fmaf(f[0], x0.x, acc0); acc0 = fmaf(f[1], x0.y, acc0);
        acc0 = fmaf(f[2], x0.z, acc0); acc0 = fmaf(f[3], x0.w, acc0);
        acc0 = fmaf(f[4], x1.x, acc0); acc0 = fmaf(f[5], x1.y, acc0);
        acc0 = fmaf(f[6], x1.z, acc0); acc0 = fmaf(f[7], x1.w, acc0);
        if (two) {
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(w1 + k0), f);
          acc1 = fmaf(f[0], x0.x, acc1); acc1 = fmaf(f[1], x0.y, acc1);
          acc1 = fmaf(f[2], x0.z, acc1); acc1 = fmaf(f[3], x0.w, acc1);
          acc1 = fmaf(f[4], x1.x, acc1); acc1 = fmaf(f[5], x1.y, acc1);
          acc1 = fmaf(f[6], x1.z, acc1); acc1 = fmaf(f[7], x1.w, acc1);
        }
      }
      v0 = warp_sum(acc0);
      v1 = warp_sum(acc1);
    }
    if (lane == 0) {
      vals[rr] = v0;
      if (two) vals[rr + 1] = v1;
    }
  }
  __syncthreads();
  tline.sub(a.tl, a.tl_count, 110);
  cluster_wait();  // every CTA of the cluster has started
  for (int t = d; t < rpc * kSplits; t += kQA) {  // this CTA's rows into every CTA's allv
    const int q = t / rpc, rr = t - q * rpc;
    *cluster.map_shared_rank(&allv[g0 + rr], q) = vals[rr];
  }
  cluster_arrive();
  cluster_wait();  // every CTA's rows have arrived
  tline.sub(a.tl, a.tl_count, 111);
  }

  // ---- phase 2: gather this head group's raw q/k/v from the cluster
  // (per-dimension work: threads 0..127, warps 0..3; the other warps wait at the barriers)
  const bool hd = d < kHd;
  float raw[MG + 2];
#pragma unroll
  for (int g = 0; g < MG + 2; ++g) {
    int gi = g < G ? g * kHd + d : (g == MG ? G * kHd + d : (g == MG + 1 ? (G + 1) * kHd + d : -1));
    if (PROJ) {
      raw[g] = hd && gi >= 0 ? allv[gi] : 0.f;
    } else {  // rows of the batched projection: q heads, then k, then v
      const int row = g < G ? (kvh * G + g) * kHd : g == MG ? (a.n_heads + kvh) * kHd : (a.n_heads + a.n_kv + kvh) * kHd;
      raw[g] = hd && gi >= 0 ? a.qkv[row + d] : 0.f;
    }
  }
  if (hd) {
#pragma unroll
    for (int g = 0; g <= MG; ++g) {
      float v = raw[g];
      float s2 = warp_sum(v * v);
      if (lane == 0 && (g < G || g == MG)) red[warp][g < G ? g : G] = s2;
    }
  }
  __syncthreads();
  float nv[MG + 1];
#pragma unroll
  for (int g = 0; g <= MG; ++g) {
    if (hd && (g < G || g == MG)) {
      int r = g < G ? g : G;
      float tot = red[0][r] + red[1][r] + red[2][r] + red[3][r];
      float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)kHd), a.eps)));
      nv[g] = __fmul_rn(__fmul_rn(raw[g], inv), g < G ? qn : kn);
      hv[g < G ? g : MG][d] = nv[g];
    }
  }
  __syncthreads();
  // NeoX rotation (generic path, kernels/mod.rs:1780-1788): pairs (d, d + 64).
  float rot[MG + 1];
#pragma unroll
  for (int g = 0; g <= MG; ++g) {
    if (hd && (g < G || g == MG)) {
      int h = g < G ? g : MG;
      if (d < kHd / 2) rot[g] = __fadd_rn(__fmul_rn(nv[g], c), __fmul_rn(-hv[h][d + kHd / 2], sn));
      else rot[g] = __fadd_rn(__fmul_rn(nv[g], c), __fmul_rn(hv[h][d - kHd / 2], sn));
    }
  }
  __syncthreads();
  if (hd) {
#pragma unroll
    for (int g = 0; g <= MG; ++g)
      if (g < G || g == MG) hv[g < G ? g : MG][d] = rot[g];
    hv[MG + 1][d] = raw[MG + 1];
  }
  if (hd && rank == 0) {
    kb[(size_t)pos * kHd + d] = rot[MG];
    vb[(size_t)pos * kHd + d] = raw[MG + 1];
  }
  __syncthreads();
  if (npre > 0) mbar_wait(&kvbar, 0, a.err, 3);
  const float* ks = hv[MG];
  const float* vs = hv[MG + 1];
  for (int vw = warp; vw < kVW; vw += kQAW) {
    float m[MG], l[MG], o[MG][4];
#pragma unroll
    for (int g = 0; g < MG; ++g) {
      m[g] = -3.0e38f;
      l[g] = 0.f;
      o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
    }
    for (int jb = j0 + vw * 4; jb < j1; jb += 4 * kVW) {
      float4 kv[4], vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = jb + u;
        if (j < j1 && j != pos) {
          if (j - j0 < npre) {
            kv[u] = reinterpret_cast<const float4*>(ksm + (size_t)(j - j0) * kHd)[lane];
            vv[u] = reinterpret_cast<const float4*>(vsm + (size_t)(j - j0) * kHd)[lane];
          } else {
            kv[u] = __ldcg(reinterpret_cast<const float4*>(kb + (size_t)j * kHd) + lane);
            vv[u] = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)j * kHd) + lane);
          }
        } else {
          kv[u] = *reinterpret_cast<const float4*>(&ks[lane * 4]);
          vv[u] = *reinterpret_cast<const float4*>(&vs[lane * 4]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (jb + u >= j1) break;
#pragma unroll
        for (int g = 0; g < MG; ++g) {
          if (g >= G) break;
          float4 q = *reinterpret_cast<const float4*>(&hv[g][lane * 4]);
          float p = q.x * kv[u].x;
          p = fmaf(q.y, kv[u].y, p);
          p = fmaf(q.z, kv[u].z, p);
          p = fmaf(q.w, kv[u].w, p);
          float sc = __fmul_rn(warp_sum(p), a.scale);
          float mn = fmaxf(m[g], sc);
          float corr = expf(__fsub_rn(m[g], mn));
          float e = expf(__fsub_rn(sc, mn));
          l[g] = fmaf(l[g], corr, e);
          o[g][0] = fmaf(o[g][0], corr, e * vv[u].x);
          o[g][1] = fmaf(o[g][1], corr, e * vv[u].y);
          o[g][2] = fmaf(o[g][2], corr, e * vv[u].z);
          o[g][3] = fmaf(o[g][3], corr, e * vv[u].w);
          m[g] = mn;
        }
      }
    }
#pragma unroll
    for (int g = 0; g < MG; ++g) {
      if (g >= G) break;
      if (lane == 0) {
        wm[vw][g] = m[g];
        wl[vw][g] = l[g];
      }
      *reinterpret_cast<float4*>(&wo[vw][g][lane * 4]) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
    }
  }
  __syncthreads();
  for (int g = 0; g < G && hd; ++g) {
    float M = wm[0][g];
#pragma unroll
    for (int w = 1; w < kVW; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kVW; ++w) {
      float f = wl[w][g] > 0.f ? expf(__fsub_rn(wm[w][g], M)) : 0.f;
      L = fmaf(wl[w][g], f, L);
      O = fmaf(wo[w][g][d], f, O);
    }
    po[g][d] = O;
    if (d == 0) {
      pm[g] = M;
      pl[g] = L;
    }
  }
  // Push this split's partial of the dims each CTA finalises (CTA q: dims [q*8, q*8 + 8) of
  // every head of the group), then one cluster barrier; nothing reads a peer afterwards.
  tline.sub(a.tl, a.tl_count, 112);
  __syncthreads();
  if (!PROJ) cluster_wait();  // every CTA of the cluster has started
  for (int i = d; i < G * kHd; i += kQA) {
    const int g = i / kHd, dim = i - g * kHd, q = dim / kDimsPerCta;
    *cluster.map_shared_rank(&rcv_o[rank][g][dim - q * kDimsPerCta], q) = po[g][dim];
  }
  if (d < G * kSplits) {
    const int g = d / kSplits, q = d - g * kSplits;
    *cluster.map_shared_rank(&rcv_m[rank][g], q) = pm[g];
    *cluster.map_shared_rank(&rcv_l[rank][g], q) = pl[g];
  }
  cluster_arrive();
  cluster_wait();
  tline.mark(3);
  if (d < G * kDimsPerCta) {
    const int g = d / kDimsPerCta, dd = d % kDimsPerCta, dim = rank * kDimsPerCta + dd;
    float Ms[kSplits], Ls[kSplits], Os[kSplits];
#pragma unroll
    for (int r = 0; r < kSplits; ++r) {
      Ms[r] = rcv_m[r][g];
      Ls[r] = rcv_l[r][g];
      Os[r] = rcv_o[r][g][dd];
    }
    float M = -3.0e38f;
#pragma unroll
    for (int r = 0; r < kSplits; ++r)
      if (Ls[r] > 0.f) M = fmaxf(M, Ms[r]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int r = 0; r < kSplits; ++r) {
      if (Ls[r] > 0.f) {
        float f = expf(__fsub_rn(Ms[r], M));
        L = fmaf(Ls[r], f, L);
        O = fmaf(Os[r], f, O);
      }
    }
    a.out[(kvh * G + g) * kHd + dim] = __fdiv_rn(O, L);
  }
}

// ------------------------------------------------------------------ host side
namespace {
// Shared memory of a streaming matvec inside the step: 160 KB of weight stages in flight per
// SM keep HBM busy (the 1.7B bf16 gate/up and down projections ran at 1.7-2.7 TB/s with the
// earlier 112 KB), at the cost of the successor's early CTAs sharing the SM only when small.
constexpr int kSmemBudget = 160 * 1024;
constexpr size_t kSmallSmemMax = 200 * 1024;
constexpr int kAttnKvRows = 16;  // K/V rows per CTA staged before the wait (attention-only kernel)
constexpr size_t kSplitSlabBytes = 64 * 1024;  // single-sequence split above this slab (1.7B bf16)

struct MvPlan {
  int grid, rows_per_cta, block_rows, nkc, stages, cps;
  size_t smem;
};

int env_int(const char* name, int dflt) {
  const char* e = getenv(name);
  return e ? atoi(e) : dflt;
}

// Streaming-matvec tuning (read once): block rows of a stage for the inner kernels (0: by
// rows per CTA), their ring-depth cap and their shared-memory budget in KB.
struct MvTune {
  int block, max_stages, budget, stage_kb;
};
const MvTune& mv_tune() {
  static const MvTune t{env_int("QASR_MV_BLOCK", 0), env_int("QASR_MV_STAGES", 12),
                        env_int("QASR_MV_BUDGET_KB", kSmemBudget / 1024),
                        env_int("QASR_MV_STAGE_KB", 64)};
  return t;
}

// norm: the kernel stages RMSNorm weights (K floats of shared memory).
MvPlan plan_mv(int N, int K, bool int8, int B, int num_sms, bool swiglu, bool last_kernel, bool norm = true) {
  MvPlan p{};
  const MvTune& tune = mv_tune();
  const int row_bytes = K * (int8 ? 1 : 2);
  const int raw = (N + num_sms - 1) / num_sms;
  p.block_rows = raw >= 48 ? 64 : (raw >= 24 || swiglu) ? 32 : 16;
  if (!last_kernel && tune.block > 0) p.block_rows = std::max(tune.block, swiglu ? 32 : 16);
  p.rows_per_cta = (raw + p.block_rows - 1) / p.block_rows * p.block_rows;
  p.grid = (N + p.rows_per_cta - 1) / p.rows_per_cta;
  p.nkc = (row_bytes + kChunk - 1) / kChunk;
  const int kpad = p.nkc * kChunk / (int8 ? 1 : 2);
  const size_t xbytes = int8 ? (size_t)kpad * 4 + (((size_t)B * kpad + 15) & ~(size_t)15) : (size_t)B * kpad * 4;
  const size_t fixed = 1024 + xbytes + 16 * 8 + (size_t)p.rows_per_cta * 4 + (norm ? (size_t)K * 4 : 0);
  // The step's last kernel (lm_head) has no successor to share the SM with: deeper ring.
  // Batched steps read each weight stage for several sequences, so they take the larger
  // budget as well (fewer resident successors matter less than the longer compute).
  const size_t budget = (last_kernel || B > 1) ? kSmallSmemMax : (size_t)tune.budget * 1024;
  // Chunks per stage: the largest divisor of nkc keeping a stage within tune.stage_kb and two
  // stages within the budget. Fewer, larger stages cut the per-stage barrier round trips that
  // bound short row blocks (the 16-row down projection: 24 stages of 8 KB otherwise).
  p.cps = 1;
  for (int c = 2; c <= p.nkc; ++c) {
    const size_t st = (size_t)p.block_rows * kChunk * c;
    if (p.nkc % c == 0 && st <= (size_t)tune.stage_kb * 1024 && fixed + 2 * st <= budget) p.cps = c;
  }
  const size_t stage = (size_t)p.block_rows * kChunk * p.cps;
  const int total = (p.rows_per_cta / p.block_rows) * (p.nkc / p.cps);
  if (fixed + 2 * stage > budget) {
    p.stages = 0;
    return p;
  }
  p.stages = (int)std::max<size_t>(2, std::min<size_t>((budget - fixed) / stage, last_kernel ? 8 : B > 1 ? 6 : tune.max_stages));
  p.stages = std::min(p.stages, std::max(total, 1));
  p.smem = (size_t)p.stages * stage + fixed;
  return p;
}

// Launch with programmatic stream serialisation (PDL) and an optional cluster shape.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                      int cluster_y, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = cluster_y;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <bool INT8, int EPI>
cudaError_t mv_launch(const CUtensorMap& map, const MvArgs& m, const MvPlan& p, cudaStream_t s, bool pdl, bool batch) {
  const int rpw = p.block_rows / kWarps;
  const dim3 g(p.grid), t(kThreads);
  if (batch) {
    if (rpw == 4) return launch_ex(mv_kernel<INT8, EPI, 4, true>, g, t, p.smem, s, pdl, 1, map, m);
    else if (rpw == 2) return launch_ex(mv_kernel<INT8, EPI, 2, true>, g, t, p.smem, s, pdl, 1, map, m);
    else return launch_ex(mv_kernel<INT8, EPI, 1, true>, g, t, p.smem, s, pdl, 1, map, m);
  } else {
    if (rpw == 4) return launch_ex(mv_kernel<INT8, EPI, 4, false>, g, t, p.smem, s, pdl, 1, map, m);
    else if (rpw == 2) return launch_ex(mv_kernel<INT8, EPI, 2, false>, g, t, p.smem, s, pdl, 1, map, m);
    else return launch_ex(mv_kernel<INT8, EPI, 1, false>, g, t, p.smem, s, pdl, 1, map, m);
  }
}

bool launched_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  set_error(std::string("decode: ") + what + " launch failed: " + cudaGetErrorString(e));
  return false;
}

// Shared memory of the single-stage small matvec for B sequences (0 when it does not apply).
size_t small_smem(int N, int K, bool int8, int B, int num_sms, int* rpc_out, int* nkc_out) {
  const int row_bytes = K * (int8 ? 1 : 2);
  const int raw = (N + num_sms - 1) / num_sms;
  const int rpc = raw + (raw & 1);
  const int nkc = (row_bytes + kChunk - 1) / kChunk;
  const int kpad = nkc * kChunk / (int8 ? 1 : 2);
  const size_t xbytes = int8 ? (size_t)kpad * 4 + (((size_t)B * kpad + 15) & ~(size_t)15) : (size_t)B * kpad * 4;
  if (rpc_out) *rpc_out = rpc;
  if (nkc_out) *nkc_out = nkc;
  return 1024 + (size_t)nkc * rpc * kChunk + xbytes + (size_t)((rpc + 3) & ~3) * 4 + (size_t)K * 4 + (size_t)B * rpc * nkc * 4 + 64;
}

// The single-stage kernel takes a matrix when each CTA's slab is at most 48 rows and at most
// 100 KB (larger slabs arrive as one batch with nothing to overlap: the streaming ring
// kernel is faster there) and its shared memory fits.
bool small_ok(int N, int K, bool int8, int B, int num_sms) {
  int rpc = 0, nkc = 0;
  const size_t smem = small_smem(N, K, int8, B, num_sms, &rpc, &nkc);
  const int raw = (N + num_sms - 1) / num_sms;
  return raw <= 48 && (size_t)nkc * rpc * kChunk <= 100 * 1024 && smem <= kSmallSmemMax;
}

// allow_small = false keeps the streaming kernel, whose f32 dot products accumulate each
// lane's chunks in order before one warp reduction (the fused QKV kernel's order).
template <int EPI>
// batch_kernels selects the batched instantiations also for B = 1 (their staging order is
// the one sum_threads names).
bool mv(bool int8, const void* W, MvArgs m, int num_sms, cudaStream_t s, bool pdl = true, bool allow_small = true,
        bool batch_kernels = false) {
  const bool batch = m.B > 1 || batch_kernels;
  const int row_bytes = m.K * (int8 ? 1 : 2);
  int rpc = 0, nkc = 0;
  const size_t smem_small = small_smem(m.N, m.K, int8, m.B, num_sms, &rpc, &nkc);
  if (EPI != MV_ARGMAX && allow_small && small_ok(m.N, m.K, int8, m.B, num_sms)) {
    // small matrix: one stage per CTA holding the whole slab, K split across warps
    m.rows_per_cta = rpc;
    m.nkc = nkc;
    CUtensorMap map;
    if (!make_tma_2d_u16(&map, W, m.N, row_bytes / 2, kChunk / 2, rpc)) {
      set_error("decode: cannot encode the weight tensor map");
      return false;
    }
    dim3 grid((m.N + rpc - 1) / rpc);
    const dim3 t(kThreads);
    cudaError_t e;
    if (batch) {
      if (int8) e = launch_ex(mv_small_batch_kernel<true, EPI>, grid, t, smem_small, s, pdl, 1, map, m);
      else e = launch_ex(mv_small_batch_kernel<false, EPI>, grid, t, smem_small, s, pdl, 1, map, m);
    } else {
      if (int8) e = launch_ex(mv_small_kernel<true, EPI>, grid, t, smem_small, s, pdl, 1, map, m);
      else e = launch_ex(mv_small_kernel<false, EPI>, grid, t, smem_small, s, pdl, 1, map, m);
    }
    return launched_ok(e, "small matvec");
  }
  MvPlan p = plan_mv(m.N, m.K, int8, m.B, num_sms, EPI == MV_SWIGLU, EPI == MV_ARGMAX, m.norm_w != nullptr);
  if (p.stages == 0) {
    set_error("decode: no ring of two stages fits the matvec shared memory");
    return false;
  }
  m.rows_per_cta = p.rows_per_cta;
  m.block_rows = p.block_rows;
  m.nkc = p.nkc;
  m.stages = p.stages;
  m.cps = p.cps;
  CUtensorMap map;
  if (!make_tma_2d_u16(&map, W, m.N, row_bytes / 2, kChunk / 2, p.block_rows)) {
    set_error("decode: cannot encode the weight tensor map");
    return false;
  }
  return launched_ok(int8 ? mv_launch<true, EPI>(map, m, p, s, pdl, batch) : mv_launch<false, EPI>(map, m, p, s, pdl, batch),
                     "streaming matvec");
}

template <bool INT8, int EPI>
void mv_attr(int bytes) {
  for (auto k : {mv_kernel<INT8, EPI, 1, false>, mv_kernel<INT8, EPI, 2, false>, mv_kernel<INT8, EPI, 4, false>,
                 mv_kernel<INT8, EPI, 1, true>, mv_kernel<INT8, EPI, 2, true>, mv_kernel<INT8, EPI, 4, true>})
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}
}  // namespace

size_t decode_staged_bytes(int hidden, int q_dim, int inter) {
  const int k = std::max(hidden, std::max(q_dim, inter));
  const size_t kpad = ((size_t)k + kChunk - 1) / kChunk * kChunk;  // >= either mode's padding
  return (size_t)kDecodeMaxBatch * kpad * 4 + 1024;
}

bool decode_stage_once() {
  static const bool on = [] {
    const char* e = getenv("QASR_STAGE_ONCE");
    return !e || atoi(e) != 0;
  }();
  return on;
}

int decode_batched_step_launches(int layers, bool int8) {
  return int8 && decode_stage_once() ? 9 * layers + 2 : 5 * layers + 1;
}

void decode_kernels_init() {
  const int kMax = 210 * 1024;
  for (auto k : {stage_kernel<true>, stage_kernel<false>})
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
  for (auto k : {mv_small_kernel<true, MV_RESID>, mv_small_kernel<false, MV_RESID>, mv_small_kernel<true, MV_STORE>,
                 mv_small_kernel<false, MV_STORE>, mv_small_kernel<true, MV_SWIGLU>,
                 mv_small_kernel<false, MV_SWIGLU>, mv_small_batch_kernel<true, MV_RESID>,
                 mv_small_batch_kernel<false, MV_RESID>, mv_small_batch_kernel<true, MV_STORE>,
                 mv_small_batch_kernel<false, MV_STORE>, mv_small_batch_kernel<true, MV_SWIGLU>,
                 mv_small_batch_kernel<false, MV_SWIGLU>})
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax);
  mv_attr<true, MV_STORE>(kMax);
  mv_attr<true, MV_RESID>(kMax);
  mv_attr<true, MV_SWIGLU>(kMax);
  mv_attr<true, MV_ARGMAX>(kMax);
  mv_attr<false, MV_STORE>(kMax);
  mv_attr<false, MV_RESID>(kMax);
  mv_attr<false, MV_SWIGLU>(kMax);
  mv_attr<false, MV_ARGMAX>(kMax);
  for (auto k : {qkv_attn_kernel<true, true, 2>, qkv_attn_kernel<false, true, 2>, qkv_attn_kernel<true, false, 2>,
                 qkv_attn_kernel<false, false, 2>, qkv_attn_kernel<true, true, kMaxG>,
                 qkv_attn_kernel<false, true, kMaxG>, qkv_attn_kernel<true, false, kMaxG>,
                 qkv_attn_kernel<false, false, kMaxG>}) {
    // its static shared memory (~22 KB) plus this stays within the 227 KB per block
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  }
}

// A single sequence also takes the split q/k/v path (batched matvec + attention-only
// kernel) when the fused kernel's per-CTA weight slab is large: each CTA of the fused kernel
// fetches (G + 2) * 128 / kSplits rows, which for 1.7B bf16 is 128 KB and arrives too late to
// overlap. Both paths give the same bits.
bool decode_split_qkv(int hidden, int q_heads, int kv_heads, bool int8) {
  static const int env = [] {
    const char* e = getenv("QASR_SPLIT_QKV");
    return e ? atoi(e) : -1;
  }();
  if (env >= 0) return env != 0;
  const size_t slab = (size_t)(q_heads / kv_heads + 2) * kHd / kSplits * hidden * (int8 ? 1 : 2);
  return slab > kSplitSlabBytes;
}

int decode_max_batch(int hidden, int inter, int q_heads, int kv_heads, bool int8) {
  const int nsm = sm_count();
  const int qd = q_heads * kHd;
  int best = 1;
  for (int B = 2; B <= kDecodeMaxBatch; ++B) {
    bool ok = true;
    // every matvec must fit either the small kernel or a streaming ring of >= 2 stages
    const int shapes[4][2] = {{hidden, qd}, {2 * inter, hidden}, {hidden, inter}, {1 << 17, hidden}};
    // the batched q/k/v projection (int8: either kernel; bf16: the streaming kernel)
    const int nqkv = qd + 2 * kv_heads * kHd;
    if (!(int8 && small_ok(nqkv, hidden, true, B, nsm)) && plan_mv(nqkv, hidden, int8, B, nsm, false, false).stages == 0)
      ok = false;
    for (int i = 0; i < 4 && ok; ++i) {
      const int N = shapes[i][0], K = shapes[i][1];
      const int raw = (N + nsm - 1) / nsm;
      auto small_at = [&](int b) {
        (void)raw;
        return i < 3 && small_ok(N, K, int8, b, nsm);
      };
      // the kernel (and so the summation order) must be the one a single sequence gets
      if (small_at(1) != small_at(B)) ok = false;
      if (!small_at(B) && plan_mv(N, K, int8, B, nsm, i == 1, i == 3).stages == 0) ok = false;
    }
    if (!ok) break;
    best = B;
  }
  return best;
}

bool decode_step(const DecodeArgs& a, cudaStream_t s) {
  static thread_local int cached_dev = -1, cached_sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    cached_dev = dev;
    cached_sms = sm_count();
  }
  const int nsm = cached_sms;
  const int B = std::max(1, a.batch);
  const int qd = a.q_heads * kHd;
  static const bool sync_check = getenv("QASR_SYNC_CHECK") != nullptr;
  auto check = [&](const char* what, int layer) {  // debugging aid: plain launches only
    if (!sync_check) return;
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) fprintf(stderr, "decode_step: %s (layer %d, batch %d): %s\n", what, layer, B, cudaGetErrorString(e));
  };
  bool ok = true;  // every launch of the step was planned and accepted
  auto launched = [&](cudaError_t e) { ok = launched_ok(e, "kernel") && ok; };
  // Batched int8 steps: each matvec's inputs staged once by stage_kernel (one CTA a
  // sequence) before it. int8 staging reads the inputs three times (norm, absmax, quantise),
  // 4-9 us per CTA-redundant pass at B = 8 (1.7B); bf16 staging is cheaper than the extra
  // kernel hand-over, so bf16 batched steps keep staging in every CTA.
  const bool pre_stage = B > 1 && a.int8 && a.staged && decode_stage_once();
  auto stage = [&](MvArgs& m, bool pdl) {
    if (!pre_stage) return;
    MvArgs sa = m;
    sa.nkc = (m.K * (a.int8 ? 1 : 2) + kChunk - 1) / kChunk;
    sa.staged = a.staged;
    sa.kind = 6;
    const int kpad = sa.nkc * kChunk / (a.int8 ? 1 : 2);
    const size_t smem = 16 + (size_t)kpad * (a.int8 ? 1 : 4) + (m.norm_w ? (size_t)m.K * 4 : 0);
    launched(launch_ex(a.int8 ? stage_kernel<true> : stage_kernel<false>, dim3(1, B), dim3(kThreads), smem, s, pdl, 1, sa));
    m.staged = a.staged;
  };
  auto run = [&](auto epi_tag, const void* W, const MvArgs& m) {
    constexpr int EPI = decltype(epi_tag)::value;
    ok = mv<EPI>(a.int8, W, m, nsm, s) && ok;
  };
  using Resid = std::integral_constant<int, MV_RESID>;
  using Swiglu = std::integral_constant<int, MV_SWIGLU>;
  using Argmax = std::integral_constant<int, MV_ARGMAX>;
  auto base = [&](int kind) {
    MvArgs m{};
    m.eps = a.eps; m.err = a.err;
    m.tl = a.tl; m.tl_count = a.tl_count; m.kind = kind;
    m.B = B;
    return m;
  };
  const bool split = B > 1 || decode_split_qkv(a.hidden, a.q_heads, a.kv_heads, a.int8);
  for (int l = 0; l < a.layers; ++l) {
    // QKV projection + attention, one cluster per (kv head, sequence). The first kernel of a
    // step is a plain launch: it starts only after the previous step (which advanced
    // StepState and wrote the last KV row) has completed, so every kernel of the step may
    // read StepState and earlier KV rows before its dependency wait.
    const int nqkv = (a.q_heads + 2 * a.kv_heads) * kHd;
    if (split) {
      // batched steps: one matvec projects q/k/v of every sequence (input RMSNorm fused,
      // staged in the fused kernel's summation order), then the attention-only kernel
      MvArgs m = base(0);
      m.x = a.x; m.ldx = a.hidden; m.st = a.st;
      if (l == 0) {
        m.embed = a.embed;
        m.x_out = a.x;
      }
      m.norm_w = a.n1[l]; m.K = a.hidden; m.N = nqkv; m.ws = a.s_qkv[l]; m.out = a.qkv; m.ldo = nqkv;
      m.sum_threads = a.int8 ? qa_threads<true>() : qa_threads<false>();
      stage(m, l != 0);  // the step's first kernel is a plain launch
      ok = mv<MV_STORE>(a.int8, a.w_qkv[l], m, nsm, s, l != 0 || pre_stage, a.int8, true) && ok;
      if (a.on_launch) a.on_launch(a.hook_ctx, 0);
      check("qkv_proj", l);
    }
    {
      QkvAttnArgs q{};
      q.x = a.x;
      if (l == 0) {
        q.embed = a.embed;
        q.x_out = a.x;
      }
      q.norm_w = a.n1[l]; q.eps = a.eps; q.K = a.hidden; q.W = a.w_qkv[l]; q.ws = a.s_qkv[l];
      q.n_heads = a.q_heads; q.n_kv = a.kv_heads; q.qn = a.qn[l]; q.kn = a.kn[l];
      q.rc = a.rope_cos; q.rs = a.rope_sin;
      q.kc = a.k_cache + (size_t)l * a.kv_heads * a.max_seq * kHd;
      q.vc = a.v_cache + (size_t)l * a.kv_heads * a.max_seq * kHd;
      q.max_seq = a.max_seq; q.scale = 1.0f / sqrtf((float)kHd);
      q.rows_per_cta = (a.q_heads / a.kv_heads + 2) * kHd / kSplits;
      q.st = a.st; q.out = a.attn; q.err = a.err; q.tl = a.tl; q.tl_count = a.tl_count;
      q.ldx = a.hidden; q.ldo = qd; q.kv_slot_stride = a.kv_slot_stride;
      const dim3 grid(a.kv_heads, kSplits, B);
      const bool g2 = a.q_heads <= 2 * a.kv_heads;  // group arrays sized for 2 q heads
      if (split) {
        q.embed = nullptr;
        q.x_out = nullptr;
        q.qkv = a.qkv;
        q.ldq = nqkv;
        q.rows_per_cta = 0;
        q.kv_rows = kAttnKvRows;
        const size_t smem = (size_t)q.kv_rows * kHd * 8;
        const dim3 t(128);
        if (g2) {
          if (a.int8) launched(launch_ex(qkv_attn_kernel<true, false, 2>, grid, t, smem, s, true, kSplits, q));
          else launched(launch_ex(qkv_attn_kernel<false, false, 2>, grid, t, smem, s, true, kSplits, q));
        } else {
          if (a.int8) launched(launch_ex(qkv_attn_kernel<true, false, kMaxG>, grid, t, smem, s, true, kSplits, q));
          else launched(launch_ex(qkv_attn_kernel<false, false, kMaxG>, grid, t, smem, s, true, kSplits, q));
        }
      } else {
        const size_t wbytes = ((size_t)q.rows_per_cta * a.hidden * (a.int8 ? 1 : 2) + 127) & ~(size_t)127;
        const size_t tail = (size_t)a.hidden * 5 + 16 + 64 * 4 + (size_t)a.hidden * 4;
        const size_t budget = 200 * 1024;
        q.kv_rows = (int)std::max<long>(0, std::min<long>(24, ((long)budget - (long)(wbytes + tail)) / (2 * kHd * 4)));
        const size_t smem = wbytes + (size_t)q.kv_rows * kHd * 8 + tail;
        const bool p = l != 0;
        if (g2) {
          if (a.int8) launched(launch_ex(qkv_attn_kernel<true, true, 2>, grid, dim3(qa_threads<true>()), smem, s, p, kSplits, q));
          else launched(launch_ex(qkv_attn_kernel<false, true, 2>, grid, dim3(qa_threads<false>()), smem, s, p, kSplits, q));
        } else {
          if (a.int8) launched(launch_ex(qkv_attn_kernel<true, true, kMaxG>, grid, dim3(qa_threads<true>()), smem, s, p, kSplits, q));
          else launched(launch_ex(qkv_attn_kernel<false, true, kMaxG>, grid, dim3(qa_threads<false>()), smem, s, p, kSplits, q));
        }
      }
      if (a.on_launch) a.on_launch(a.hook_ctx, 1);
      check("qkv_attn", l);
    }
    // O projection + residual
    MvArgs m = base(2);
    m.x = a.attn; m.ldx = qd; m.K = qd; m.N = a.hidden;
    m.ws = a.s_o[l]; m.out = a.x; m.resid = a.x; m.ldo = a.hidden;
    stage(m, true);
    run(Resid{}, a.w_o[l], m);
    if (a.on_launch) a.on_launch(a.hook_ctx, 2);
    check("o_proj", l);
    // gate/up (post-attention RMSNorm fused) + SwiGLU
    m = base(3);
    m.x = a.x; m.ldx = a.hidden; m.norm_w = a.n2[l]; m.K = a.hidden; m.N = 2 * a.inter;
    m.ws = a.s_gu[l]; m.out = a.ffn; m.ldo = a.inter;
    stage(m, true);
    run(Swiglu{}, a.w_gu[l], m);
    if (a.on_launch) a.on_launch(a.hook_ctx, 3);
    check("gate_up", l);
    // down projection + residual
    m = base(4);
    m.x = a.ffn; m.ldx = a.inter; m.K = a.inter; m.N = a.hidden;
    m.ws = a.s_down[l]; m.out = a.x; m.resid = a.x; m.ldo = a.hidden;
    stage(m, true);
    run(Resid{}, a.w_down[l], m);
    if (a.on_launch) a.on_launch(a.hook_ctx, 4);
    check("down", l);
  }
  MvArgs m = base(5);
  m.x = a.x; m.ldx = a.hidden; m.norm_w = a.final_norm; m.K = a.hidden; m.N = a.vocab;
  m.ws = a.lm_s;
  m.am_part = a.am_part; m.am_ticket = a.am_ticket; m.st = a.st; m.tokens = a.tokens; m.forced = a.forced;
  m.tokens_ld = a.tokens_ld;
  m.logits = a.logits;
  stage(m, true);
  run(Argmax{}, a.lm_w, m);
  if (a.on_launch) a.on_launch(a.hook_ctx, 5);
  check("lm_head", -1);
  return ok;
}

}  // namespace qasr
