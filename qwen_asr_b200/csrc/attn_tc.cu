// Tensor-core attention for sm_100a (tcgen05.mma with TMEM accumulators): the encoder's
// windowed bidirectional attention (kernels/mod.rs:1386-1474, windows from
// encoder.rs:292-298) and the decoder prefill's causal GQA attention over the f32 KV cache
// (kernels/mod.rs:1480-1701 with a start offset, decoder.rs:455-547).
//
// One CTA (256 threads) owns up to 128 queries of one head. Query row r is TMEM lane r; the
// two warps of lane quarter r / 32 each take half of the row's score columns and half of its
// output dims, and combine row maxima and sums through shared memory (sums in a fixed order).
// Keys go in blocks of BK:
//   S = Q K^T  (tcgen05, M = 128, N = BK, K = D)  -> TMEM columns [0, BK)
//   p = exp(S * scale - m), running max m and sum l per row (online softmax, as the
//       reference's single-pass loop; masked keys get p = 0)
//   O_blk = P V (tcgen05, M = 128, N = D, K = BK)   -> TMEM columns [BK, BK + D)
//   O = O * corr + O_blk in registers; at the end O / l (the reference's 1 / sum_exp scale).
// Precision. q, k, v and p are f32. Each enters the MMAs as three bf16 planes
// (x = hi + mid + lo, split3_bf16), and the six plane products whose weight is >= 2^-16 of the
// leading one (hi*hi, hi*mid, mid*hi, hi*lo, mid*mid, lo*hi) are accumulated in f32, so
// scores and outputs carry f32-level error like the reference's f32 dot products.
// Operands are staged by the threads from global memory into shared memory in the K-major
// 128-byte-swizzle layout tcgen05 reads (the layout TMA's SWIZZLE_128B writes); the
// generic-proxy writes are made visible to the tensor core with fence.proxy.async. Every wait
// on the MMA-completion barrier is bounded (an error code, never a hang).
#include <algorithm>
#include <cstdlib>
#include <vector>

#include "bulk.cuh"
#include "common.h"
#include "dev_util.cuh"
#include "kernels.h"

namespace qasr {
namespace {

constexpr int kThreads = 256, BQ = 128;
// floats per query row of a split partial: 128 output dims, the row max and the row sum,
// padded to a multiple of 4 (float4 stores)
constexpr int kPartRow = 132;

// K-major SW128 operand of R rows x C columns (bf16), three planes: plane p, 64-column chunk c
// is an R x 128-byte block at (p * C / 64 + c) * R * 128; 16-byte unit u of row r sits at
// r * 128 + ((u ^ (r & 7)) << 4).
__device__ __forceinline__ uint32_t sw_off(int R, int C, int p, int r, int col) {
  const int c = col >> 6, u = (col & 63) >> 3;
  return (uint32_t)(((p * (C >> 6) + c) * R + r) * 128 + ((u ^ (r & 7)) << 4) + ((col & 7) << 1));
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// Descriptor of plane p at K offset k (a multiple of 16 elements).
__device__ __forceinline__ uint64_t op_desc(uint32_t base, int R, int C, int p, int k) {
  return sw128_desc(base + (uint32_t)((p * (C >> 6) + (k >> 6)) * R * 128 + ((k & 63) >> 3) * 16));
}

template <int M, int N>
struct Idesc {  // kind::f16, f32 accumulator, bf16 A and B, both K-major
  static constexpr uint32_t value =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
};

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

#define TMEM_LD32(taddr, r)                                                                                       \
  asm volatile(                                                                                                   \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                              \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),           \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),     \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),   \
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])    \
      : "r"(taddr))

// Plane pairs (A plane, B plane) of the six retained products.
__constant__ int kPairA[6] = {2, 1, 0, 1, 0, 0};
__constant__ int kPairB[6] = {0, 1, 2, 0, 1, 0};

// Stages rows [0, rows) of an R x D f32 operand (row r at src + r * ld, rows >= valid are
// zero) as three K-major planes; four consecutive columns per thread-iteration, coalesced.
template <int R, int D>
__device__ __forceinline__ void stage_rows(unsigned char* dst, const float* src, long ld, int valid) {
  constexpr int G = D / 4, N = R * G / kThreads, U = N < 8 ? N : 8;  // float4s per thread, batch
  static_assert(N % U == 0, "staging batch");
#pragma unroll 1
  for (int b = 0; b < N; b += U) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {  // every load of the batch in flight before the first use
      const int idx = threadIdx.x + (b + u) * kThreads, r = idx / G, col = (idx % G) * 4;
      v[u] = r < valid ? *reinterpret_cast<const float4*>(src + (long)r * ld + col) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = threadIdx.x + (b + u) * kThreads, r = idx / G, col = (idx % G) * 4;
      const float f[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      __nv_bfloat16 h[4], m[4], l[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) split3_bf16(f[j], h[j], m[j], l[j]);
      *reinterpret_cast<uint2*>(dst + sw_off(R, D, 0, r, col)) = *reinterpret_cast<uint2*>(h);
      *reinterpret_cast<uint2*>(dst + sw_off(R, D, 1, r, col)) = *reinterpret_cast<uint2*>(m);
      *reinterpret_cast<uint2*>(dst + sw_off(R, D, 2, r, col)) = *reinterpret_cast<uint2*>(l);
    }
  }
}

// Stages V rows [0, BK) (row j at src + j * ld, rows >= valid are zero) transposed: the B
// operand of P V is [D rows = dims][BK columns = keys]. Each thread-iteration reads one dim
// of 8 consecutive keys (a warp reads 32 consecutive dims: coalesced) and writes 16 bytes.
template <int BK, int D>
__device__ __forceinline__ void stage_vt(unsigned char* dst, const float* src, long ld, int valid) {
  constexpr int N = D * (BK / 8) / kThreads;  // (dim, 8 keys) items per thread
#pragma unroll 1
  for (int b = 0; b < N; b += 2) {
    float v[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {  // 16 loads in flight
      const int idx = threadIdx.x + (b + u) * kThreads, d = idx % D, j0 = (idx / D) * 8;
#pragma unroll
      for (int t = 0; t < 8; ++t) v[u][t] = (j0 + t < valid) ? src[(long)(j0 + t) * ld + d] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int idx = threadIdx.x + (b + u) * kThreads, d = idx % D, j0 = (idx / D) * 8;
      __align__(16) __nv_bfloat16 h[8], m[8], l[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) split3_bf16(v[u][t], h[t], m[t], l[t]);
      *reinterpret_cast<uint4*>(dst + sw_off(D, BK, 0, d, j0)) = *reinterpret_cast<uint4*>(h);
      *reinterpret_cast<uint4*>(dst + sw_off(D, BK, 1, d, j0)) = *reinterpret_cast<uint4*>(m);
      *reinterpret_cast<uint4*>(dst + sw_off(D, BK, 2, d, j0)) = *reinterpret_cast<uint4*>(l);
    }
  }
}

// A prefill work item: queries [q0, q0 + nq) of the packed rows (KV positions qpos0..) of one
// sequence against its keys [kb0, kb1). A query tile whose keys span several chunks is split
// over several items (split / nsplit of one group); the last item of the group to finish
// merges the partials in split order.
struct AttnItem {
  int q0, nq, qpos0, kb0, kb1, split, nsplit, group;
  long long kv_off;   // floats from the layer's slot-0 K/V base to this sequence's slot
  long long ws_off;   // floats into the partial workspace of this group (head 0, split 0)
};

struct AttnArgs {
  const float* q;  // query row i of head h: q + i * ldq + h * D
  long ldq;
  const float* k;  // key row j of kv head g: k + g * kv_head_stride + j * ldk
  const float* v;
  long ldk, kv_head_stride;
  int heads_per_kv;
  float* out;  // out + i * ldo + h * D
  long ldo;
  __nv_bfloat16* planes;  // optional: out also as bf16 planes [3][plane], rows of ldo
  long long plane;
  float scale;
  // encoder: windows (blockIdx.x = window); prefill: query tiles of BQ rows, causal
  const int* win;  // window starts [n_win + 1] (encoder)
  int n_q, start;  // prefill: query count and the KV position of query 0
  const AttnItem* items;  // prefill: blockIdx.x -> work item (all jobs of a layer in one launch)
  long long kv_layer_off; // floats from a.k / a.v to this layer of slot 0
  float* ws;              // split partials: [BQ rows][D + 2] (O, m, l) per (group, head, split)
  int* tickets;           // [group][head], zero at rest
  int* err;
  unsigned long long* tl;  // optional timeline (debug): CTA (0, 0) thread 0 stamps phases
};

template <int D, int BK, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const AttnArgs a) {
  constexpr int kQBytes = 3 * BQ * D * 2, kKVBytes = 3 * BK * D * 2, kPBytes = 3 * BQ * BK * 2;
  constexpr int kCols = BK + D <= 128 ? 128 : 256;
  constexpr int SH = BK / 2, DH = D / 2;  // score columns and output dims of one warp
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sQ = smem;
  unsigned char* sKV = sQ + kQBytes;
  unsigned char* sP = sKV + kKVBytes;
  float* red_max = reinterpret_cast<float*>(sP + kPBytes);  // [2][BQ]: per column half
  float* red_sum = red_max + 2 * BQ;                        // [2][BQ]
  uint64_t* bar = reinterpret_cast<uint64_t*>(red_sum + 2 * BQ);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, h = blockIdx.y;
  // warps w and w + 4 share TMEM lane quarter w % 4 (query rows); half = which column half
  const int quarter = warp & 3, half = warp >> 2, row = quarter * 32 + lane;
  const int kvh = h / a.heads_per_kv;

  // this CTA's queries and keys
  int q0, nq, k0, nk, qpos0;
  AttnItem item{};
  long long kv_off = 0;
  if (CAUSAL) {
    item = a.items[blockIdx.x];
    q0 = item.q0;
    nq = item.nq;
    qpos0 = item.qpos0;  // KV position of query row 0 of the tile
    k0 = item.kb0;       // this item's keys [kb0, kb1) of the sequence's 0 .. last query position
    nk = item.kb1 - item.kb0;
    kv_off = a.kv_layer_off + item.kv_off;
  } else {
    q0 = a.win[blockIdx.x];
    nq = a.win[blockIdx.x + 1] - q0;
    k0 = q0;
    nk = nq;
    qpos0 = 0;
  }
  if (nq <= 0) return;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  unsigned long long* tl = (a.tl && blockIdx.x == gridDim.x - 1 && blockIdx.y == 0 && tid == 0) ? a.tl : nullptr;
  int ti = 0;
  if (tl) tl[ti++] = global_timer_ns();
  const float* qsrc = a.q + (long)q0 * a.ldq + (long)h * D;
  stage_rows<BQ, D>(sQ, qsrc, a.ldq, nq);
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
  const uint32_t uQ = smem_u32(sQ), uKV = smem_u32(sKV), uP = smem_u32(sP);

  const float* kbase = a.k + kv_off + (long)kvh * a.kv_head_stride + (long)k0 * a.ldk;
  const float* vbase = a.v + kv_off + (long)kvh * a.kv_head_stride + (long)k0 * a.ldk;
  const int my_last = CAUSAL ? qpos0 + row - k0 : nk - 1;  // last key (relative to k0) this row may see
  float o[DH];
#pragma unroll
  for (int d = 0; d < DH; ++d) o[d] = 0.f;
  float m_run = -1e30f, l_run = 0.f;
  uint32_t phase = 0;
  bool ok = true;

  for (int kb = 0; kb < nk && ok; kb += BK) {
    const int valid = min(BK, nk - kb);
    // ---- S = Q K^T
    if (tl && ti < 60) tl[ti++] = global_timer_ns();
    stage_rows<BK, D>(sKV, kbase + (long)kb * a.ldk, a.ldk, valid);
    if (tl && ti < 60) tl[ti++] = global_timer_ns();
    fence_async_smem();
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;");
      bool first = true;
      for (int pr = 0; pr < 6; ++pr)
#pragma unroll
        for (int kk = 0; kk < D; kk += 16) {
          mma_bf16(tmem, op_desc(uQ, BQ, D, kPairA[pr], kk), op_desc(uKV, BK, D, kPairB[pr], kk),
                   Idesc<BQ, BK>::value, first ? 0u : 1u);
          first = false;
        }
      mma_commit(bar);
    }
    ok = __syncthreads_and(mbar_wait(bar, phase, a.err, 21)) != 0;
    phase ^= 1u;
    if (tl && ti < 60) tl[ti++] = global_timer_ns();
    asm volatile("tcgen05.fence::after_thread_sync;");
    // ---- online softmax: this warp's half of the row's scores
    float s[SH];
#pragma unroll
    for (int c = 0; c < SH; c += 32) {
      uint32_t r[32];
      TMEM_LD32(trow + (uint32_t)(half * SH + c), r);
      asm volatile("tcgen05.wait::ld.sync.aligned;");
#pragma unroll
      for (int j = 0; j < 32; ++j) s[c + j] = __uint_as_float(r[j]);
    }
    const int kj0 = kb + half * SH;  // key index of s[0]
    float m_part = -1e30f;
#pragma unroll
    for (int j = 0; j < SH; ++j) {
      const bool vis = (kj0 + j < nk) && (kj0 + j <= my_last);
      s[j] = vis ? __fmul_rn(s[j], a.scale) : -INFINITY;
      m_part = fmaxf(m_part, s[j]);
    }
    red_max[half * BQ + row] = m_part;
    __syncthreads();
    const float m_new = fmaxf(m_run, fmaxf(red_max[row], red_max[BQ + row]));
    const float corr = expf(__fsub_rn(m_run, m_new));
    float psum = 0.f;
#pragma unroll
    for (int j = 0; j < SH; ++j) {
      s[j] = s[j] == -INFINITY ? 0.f : expf(__fsub_rn(s[j], m_new));
      psum = __fadd_rn(psum, s[j]);
    }
    red_sum[half * BQ + row] = psum;
    m_run = m_new;
    // P planes (this warp's columns of the row) and V^T planes (S is complete: K is free)
#pragma unroll
    for (int j0 = 0; j0 < SH; j0 += 8) {
      __align__(16) __nv_bfloat16 ph[8], pm[8], pl[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) split3_bf16(s[j0 + t], ph[t], pm[t], pl[t]);
      const int col = half * SH + j0;
      *reinterpret_cast<uint4*>(sP + sw_off(BQ, BK, 0, row, col)) = *reinterpret_cast<uint4*>(ph);
      *reinterpret_cast<uint4*>(sP + sw_off(BQ, BK, 1, row, col)) = *reinterpret_cast<uint4*>(pm);
      *reinterpret_cast<uint4*>(sP + sw_off(BQ, BK, 2, row, col)) = *reinterpret_cast<uint4*>(pl);
    }
    if (tl && ti < 60) tl[ti++] = global_timer_ns();
    stage_vt<BK, D>(sKV, vbase + (long)kb * a.ldk, a.ldk, valid);
    if (tl && ti < 60) tl[ti++] = global_timer_ns();
    fence_async_smem();
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    // row sum in a fixed order (half 0 + half 1): both warps of a row keep the same l
    l_run = __fadd_rn(__fmul_rn(l_run, corr), __fadd_rn(red_sum[row], red_sum[BQ + row]));
    // ---- O_blk = P V
    if (tid == 0 && ok) {
      asm volatile("tcgen05.fence::after_thread_sync;");
      bool first = true;
      for (int pr = 0; pr < 6; ++pr)
#pragma unroll
        for (int kk = 0; kk < BK; kk += 16) {
          mma_bf16(tmem + BK, op_desc(uP, BQ, BK, kPairA[pr], kk), op_desc(uKV, D, BK, kPairB[pr], kk),
                   Idesc<BQ, D>::value, first ? 0u : 1u);
          first = false;
        }
      mma_commit(bar);
    }
    if (ok) ok = __syncthreads_and(mbar_wait(bar, phase, a.err, 22)) != 0;
    phase ^= 1u;
    if (tl && ti < 60) tl[ti++] = global_timer_ns();
    asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
    for (int c = 0; c < DH; c += 32) {
      uint32_t r[32];
      TMEM_LD32(trow + (uint32_t)(BK + half * DH + c), r);
      asm volatile("tcgen05.wait::ld.sync.aligned;");
#pragma unroll
      for (int j = 0; j < 32; ++j) o[c + j] = __fadd_rn(__fmul_rn(o[c + j], corr), __uint_as_float(r[j]));
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();  // the next block's operands overwrite sKV / sP and its MMAs reuse TMEM
  }

  if (tl && ti < 63) tl[ti++] = global_timer_ns();
  __shared__ int s_last;
  bool merged = false;
  if (CAUSAL && item.nsplit > 1) {
    // partial (O unnormalised, m, l) of this split; the last split of the group merges
    constexpr int kRow = kPartRow;  // D dims + m + l, padded so every row starts 16-byte aligned
    static_assert(D + 2 <= kPartRow, "partial row");
    float* wp = a.ws + item.ws_off + ((long long)h * item.nsplit + item.split) * (BQ * kRow) + (long)row * kRow;
    if (ok && row < nq) {
#pragma unroll
      for (int d = 0; d < DH; d += 4)
        *reinterpret_cast<float4*>(wp + half * DH + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
      if (half == 0) {
        wp[D] = m_run;
        wp[D + 1] = l_run;
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.tickets + item.group * gridDim.y + h, 1) == item.nsplit - 1;
    __syncthreads();
    if (!s_last) {
      ok = false;  // another split of the group writes the output
    } else {
      __threadfence();
      if (row < nq) {
        const float* w0 = a.ws + item.ws_off + (long long)h * item.nsplit * (BQ * kRow) + (long)row * kRow;
        float mx = -1e30f;
        for (int sp = 0; sp < item.nsplit; ++sp) mx = fmaxf(mx, __ldcg(w0 + (long long)sp * BQ * kRow + D));
        float l = 0.f;
#pragma unroll
        for (int d = 0; d < DH; ++d) o[d] = 0.f;
        for (int sp = 0; sp < item.nsplit; ++sp) {
          const float* ws = w0 + (long long)sp * BQ * kRow;
          const float c = expf(__fsub_rn(__ldcg(ws + D), mx));
          l = __fadd_rn(l, __fmul_rn(__ldcg(ws + D + 1), c));
#pragma unroll
          for (int d = 0; d < DH; ++d) o[d] = __fadd_rn(o[d], __fmul_rn(__ldcg(ws + half * DH + d), c));
        }
        l_run = l;
      }
      __syncthreads();
      if (tid == 0) a.tickets[item.group * gridDim.y + h] = 0;  // ready for the next launch
      merged = true;
    }
  }
  (void)merged;
  if (ok && row < nq) {
    const float inv = l_run > 0.f ? __fdiv_rn(1.0f, l_run) : 0.f;
    float* orow = a.out + (long)(q0 + row) * a.ldo + (long)h * D + half * DH;
    __nv_bfloat16* prow = a.planes ? a.planes + (long)(q0 + row) * a.ldo + (long)h * D + half * DH : nullptr;
#pragma unroll
    for (int d = 0; d < DH; d += 4) {
      float4 v = make_float4(__fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv), __fmul_rn(o[d + 2], inv),
                             __fmul_rn(o[d + 3], inv));
      *reinterpret_cast<float4*>(orow + d) = v;
      if (prow) {
        const float f[4] = {v.x, v.y, v.z, v.w};
        __nv_bfloat16 hh[4], mm[4], ll[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) split3_bf16(f[j], hh[j], mm[j], ll[j]);
        *reinterpret_cast<uint2*>(prow + d) = *reinterpret_cast<uint2*>(hh);
        *reinterpret_cast<uint2*>(prow + a.plane + d) = *reinterpret_cast<uint2*>(mm);
        *reinterpret_cast<uint2*>(prow + 2 * a.plane + d) = *reinterpret_cast<uint2*>(ll);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
}

template <int D, int BK, bool CAUSAL>
constexpr int attn_smem() {
  return 1024 + 3 * BQ * D * 2 + 3 * BK * D * 2 + 3 * BQ * BK * 2 + 4 * BQ * 4 + 64;
}

int* g_attn_err[16] = {};
unsigned long long* g_attn_tl = nullptr;

int* attn_err() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16) return nullptr;
  if (!g_attn_err[dev]) {
    if (cudaMalloc(&g_attn_err[dev], sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(g_attn_err[dev], 0, sizeof(int));
    cudaFuncSetAttribute(attn_tc_kernel<64, 128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         attn_smem<64, 128, false>());
    cudaFuncSetAttribute(attn_tc_kernel<128, 64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         attn_smem<128, 64, true>());
  }
  return g_attn_err[dev];
}

}  // namespace

bool window_attention_tc(const float* qkv, float* out, __nv_bfloat16* planes, long long plane, int d, int n_heads,
                         int head_dim, const int* win_starts, int n_windows, int max_win, float scale,
                         cudaStream_t s) {
  if (head_dim != 64 || max_win > BQ || n_windows <= 0) return false;
  int* err = attn_err();
  if (!err) return false;
  AttnArgs a{};
  a.q = qkv; a.ldq = 3L * d;
  a.k = qkv + d; a.v = qkv + 2L * d; a.ldk = 3L * d; a.kv_head_stride = 64; a.heads_per_kv = 1;
  a.out = out; a.ldo = d; a.planes = planes; a.plane = plane; a.scale = scale;
  a.win = win_starts; a.err = err; a.tl = g_attn_tl;
  attn_tc_kernel<64, 128, false><<<dim3(n_windows, n_heads), kThreads, attn_smem<64, 128, false>(), s>>>(a);
  return true;
}

namespace {
struct PlanBufs {
  AttnItem* items = nullptr;
  size_t items_cap = 0;
  float* ws = nullptr;
  size_t ws_cap = 0;
  int* tickets = nullptr;
  size_t tickets_cap = 0;
};
PlanBufs g_plan[16];

template <typename T>
bool grow_buf(T*& p, size_t& cap, size_t need, bool zero) {
  if (p && cap >= need) return true;
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
  need = std::max<size_t>(need, 1024);
  if (cudaMalloc(&p, need * sizeof(T)) != cudaSuccess) {
    p = nullptr;
    return false;
  }
  if (zero && cudaMemset(p, 0, need * sizeof(T)) != cudaSuccess) return false;
  cap = need;
  return true;
}
}  // namespace

// Keys per split of a query tile (QASR_ATTN_KEY_CHUNK overrides, a multiple of 64).
static int attn_key_chunk() {
  static const int v = [] {
    const char* e = getenv("QASR_ATTN_KEY_CHUNK");
    const int c = e ? atoi(e) : kAttnKeyChunk;
    return c >= 64 ? c / 64 * 64 : kAttnKeyChunk;
  }();
  return v;
}

bool prefill_attention_plan(const std::vector<AttnBlock>& blocks, int n_heads, size_t kv_slot_stride,
                            cudaStream_t s, AttnPlan& plan) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16 || !attn_err()) return false;
  std::vector<AttnItem> items;
  long long ws = 0;
  int groups = 0;
  for (const AttnBlock& b : blocks) {
    for (int t0 = 0; t0 < b.S; t0 += BQ) {
      const int nq = std::min(BQ, b.S - t0), qpos0 = b.start + t0, kend = qpos0 + nq;
      const int chunk = attn_key_chunk();
      const int nsplit = (kend + chunk - 1) / chunk;
      for (int sp = 0; sp < nsplit; ++sp) {
        AttnItem it{};
        it.q0 = b.off + t0;
        it.nq = nq;
        it.qpos0 = qpos0;
        it.kb0 = sp * chunk;
        it.kb1 = std::min(kend, it.kb0 + chunk);
        it.split = sp;
        it.nsplit = nsplit;
        it.group = groups;
        it.kv_off = (long long)b.slot * (long long)kv_slot_stride;
        it.ws_off = ws;
        items.push_back(it);
      }
      if (nsplit > 1) ws += (long long)n_heads * nsplit * BQ * kPartRow;
      ++groups;
    }
  }
  PlanBufs& pb = g_plan[dev];
  // growing frees buffers a previous launch may still read: wait for the stream first
  if (pb.items_cap < items.size() || pb.ws_cap < (size_t)ws + 1 || pb.tickets_cap < (size_t)groups * n_heads)
    cudaStreamSynchronize(s);
  if (!grow_buf(pb.items, pb.items_cap, items.size(), false) || !grow_buf(pb.ws, pb.ws_cap, (size_t)ws + 1, false) ||
      !grow_buf(pb.tickets, pb.tickets_cap, (size_t)groups * n_heads, true))
    return false;
  if (!items.empty() &&
      cudaMemcpyAsync(pb.items, items.data(), items.size() * sizeof(AttnItem), cudaMemcpyHostToDevice, s) != cudaSuccess)
    return false;
  plan.items = pb.items;
  plan.n_items = (int)items.size();
  plan.ws = pb.ws;
  plan.tickets = pb.tickets;
  return true;
}

bool prefill_attention_tc(const AttnPlan& plan, const float* qkv, int n_heads, int n_kv, const float* kc,
                          const float* vc, long long kv_layer_off, int max_seq, float scale, float* out,
                          __nv_bfloat16* planes, long long plane, cudaStream_t s) {
  if (plan.n_items <= 0) return true;
  int* err = attn_err();
  if (!err) return false;
  const int qd = n_heads * 128, kvd = n_kv * 128;
  AttnArgs a{};
  a.q = qkv; a.ldq = qd + 2L * kvd;
  a.k = kc; a.v = vc; a.ldk = 128; a.kv_head_stride = (long)max_seq * 128; a.heads_per_kv = n_heads / n_kv;
  a.out = out; a.ldo = qd; a.planes = planes; a.plane = plane; a.scale = scale;
  a.items = (const AttnItem*)plan.items; a.kv_layer_off = kv_layer_off; a.ws = plan.ws; a.tickets = plan.tickets;
  a.err = err; a.tl = g_attn_tl;
  attn_tc_kernel<128, 64, true><<<dim3(plan.n_items, n_heads), kThreads, attn_smem<128, 64, true>(), s>>>(a);
  return true;
}

void attn_tc_set_timeline(unsigned long long* dev_buf) { g_attn_tl = dev_buf; }

int attn_tc_error() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16 || !g_attn_err[dev]) return 0;
  int e = 0;
  cudaMemcpy(&e, g_attn_err[dev], sizeof(int), cudaMemcpyDeviceToHost);
  if (e) cudaMemset(g_attn_err[dev], 0, sizeof(int));
  return e;
}

}  // namespace qasr
