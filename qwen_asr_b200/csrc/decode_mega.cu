// Persistent single-launch decode step for one sequence (Q/decoder.rs:550-645 for every
// layer, then the greedy argmax of Q/transcribe.rs:192-226).
//
// One CTA per SM (cooperative launch, so every CTA is resident), 17 warps:
//  * warp 16 is the producer: one elected lane streams, in the step's fixed order, every
//    weight tile this CTA needs (its slab of rows of qkv, o, gate/up, down for each layer,
//    then lm_head; 2-D TMA boxes of up to 32 rows x 512 bytes) and the earlier K/V rows of
//    its attention work item (1-D bulk copies) through a ring of 16 KB shared-memory slots.
//    Weights and older K/V rows do not depend on this step's activations, so the producer
//    runs ahead across phase boundaries, bounded only by the ring.
//  * warps 0..15 are consumers. Per layer they run five phases separated by grid barriers:
//    QKV projection (input RMSNorm fused), attention (q/k RMSNorm, RoPE, KV append, split
//    online-softmax over a chunk of positions; the last split of a kv head to finish merges
//    that head), O projection + residual, gate/up + SwiGLU (post-attention RMSNorm fused),
//    down projection + residual; then lm_head + argmax, whose last CTA commits the token.
// Arithmetic follows the multi-kernel path's conventions: the input vector of a matvec is
// staged in shared memory (RMSNorm with a 512-thread block sum, per-vector int8
// quantisation, kernels/mod.rs:1795-1802), and a row's value is the in-order sum of its
// 512-byte chunk dot products (int8: exact dp4a sums scaled by x_scale * w_scale).
// Every wait (mbarrier, grid barrier) is bounded: on a timeout the CTA records an error
// code, raises a global abort flag that ends every other wait at once, and runs to the end.
#include <cooperative_groups.h>
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <vector>

#include "bulk.cuh"
#include "common.h"
#include "dev_util.cuh"
#include "kernels.h"

namespace qasr {
namespace {

constexpr int kCons = 512;          // consumer threads (16 warps)
constexpr int kConsWarps = kCons / 32;
constexpr int kThr = kCons + 32;    // + the producer warp
constexpr int kSlot = 16384;        // ring slot: up to 32 rows x 512 bytes
constexpr int kChunkB = 512;        // bytes of a weight row per tile
constexpr int kTileRows = 32;
constexpr int kHdM = 128;
constexpr int kMaxGq = 4;           // q heads per kv head
constexpr int kMaxNkc = 24;         // 512-byte chunks per row
constexpr int kKvRows = 16;         // K + V rows per attention tile (8 KB each)
constexpr int kApart = kHdM + 2;    // o[128], m, l

enum { T_QKV = 0, T_O = 1, T_GU = 2, T_DOWN = 3, T_LM = 4 };

struct MegaPlan {
  int N[5], K[5], rpc[5], R[5], nkc[5];
  int splits;  // attention work items per kv head
  int nslots;
  int kpad;    // staging length (elements), >= every type's nkc * elements per chunk
  int smem;
};

struct MegaArgs {
  int H, QH, KVH, I, V, L;
  float eps;
  int int8;
  const CUtensorMap* maps;      // [L*4 + 1] in global memory
  const float* const* wscale;   // [L*4 + 1] int8 row scales
  const float* const* lnorm;    // [L*4]: n1, n2, qn, kn of each layer
  const float* final_norm;
  const __nv_bfloat16* embed;
  const float* rope_cos;
  const float* rope_sin;
  float* k_cache;
  float* v_cache;
  int max_seq;
  float* x;
  float* qkv;
  float* attn;
  float* ffn;
  float* apart;                 // [KVH][splits][kMaxGq][kApart]
  unsigned* head_ticket;        // [KVH], zero at rest
  unsigned long long* am_part;  // [grid]
  unsigned* am_ticket;          // zero at rest
  unsigned* gbar;               // [0] arrivals, [1] generation, [2] abort
  StepState* st;
  int* tokens;
  const int* forced;
  float* logits;
  int* err;
  unsigned long long* tl;       // optional timeline: CTA 0 appends {kind, t0, t1, t2}
  unsigned long long* bar_last; // [64] timeline only: arrival time of each barrier's last CTA
  int* tl_count;
  MegaPlan p;
};

// Timeline records of CTA 0 (kind: 10 + phase for a phase {start, staged, end}; 20 for a
// grid barrier {arrive, -, leave}).
struct MegaTimeline {
  unsigned long long* slot = nullptr;
  __device__ __forceinline__ void open(const MegaArgs& a, int kind) {
    slot = nullptr;
    if (a.tl && blockIdx.x == 0 && threadIdx.x == 0) {
      slot = a.tl + 4 * (size_t)atomicAdd(a.tl_count, 1);
      slot[0] = (unsigned long long)kind;
      slot[1] = slot[2] = global_timer_ns();
    }
  }
  __device__ __forceinline__ void mark(int i) {
    if (slot) slot[i] = global_timer_ns();
  }
};

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCons) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Sets the error code and the global abort flag (first failure wins the code).
__device__ __forceinline__ void mega_fail(const MegaArgs& a, volatile int* s_abort, int code) {
  atomicCAS(a.err, 0, code);
  atomicExch(a.gbar + 2, 1u);
  *s_abort = 1;
}

// Bounded mbarrier wait that also gives up as soon as an abort is raised.
__device__ bool ring_wait(const MegaArgs& a, uint64_t* b, uint32_t parity, volatile int* s_abort, int code) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 127) == 0) {
      if (*s_abort) return false;
      if (global_timer_ns() - t0 > 2000000000ull) {
        mega_fail(a, s_abort, code);
        return false;
      }
    }
  }
}

// Warp-level ring wait: lane 0 polls, the warp proceeds together.
__device__ __forceinline__ void warp_ring_wait(const MegaArgs& a, uint64_t* b, uint32_t parity, volatile int* s_abort,
                                               int code) {
  if ((threadIdx.x & 31) == 0) ring_wait(a, b, parity, s_abort, code);
  __syncwarp();
}

// Grid-wide barrier among the consumer warps of every CTA (generation counter).
__device__ void grid_sync(const MegaArgs& a, volatile int* s_abort, int code) {
  MegaTimeline tl;
  tl.open(a, 20);
  cons_sync();
  unsigned g = 0;
  if (threadIdx.x == 0 && !*s_abort) {
    unsigned* cnt = a.gbar;
    unsigned* gen = a.gbar + 1;
    g = ld_acquire(gen);
    const unsigned old = atom_add_acq_rel(cnt, 1u);
    if (old == gridDim.x - 1) {
      if (a.tl) a.bar_last[g & 63u] = global_timer_ns();
      *reinterpret_cast<volatile unsigned*>(cnt) = 0u;
      st_release(gen, g + 1u);
    } else {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire(gen) != g) break;
        if ((i & 63) == 0) {
          if (ld_acquire(a.gbar + 2)) {
            *s_abort = 1;
            break;
          }
          if (global_timer_ns() - t0 > 2000000000ull) {
            mega_fail(a, s_abort, code);
            break;
          }
        }
      }
    }
  }
  cons_sync();
  tl.mark(3);
  if (tl.slot) tl.slot[2] = __ldcg(a.bar_last + (g & 63u));
}

// Consumer block sum with block_sum's combination order for 16 warps.
__device__ __forceinline__ float cons_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  cons_sync();
  if (lane == 0) red[w] = v;
  cons_sync();
  return warp_sum(lane < kConsWarps ? red[lane] : 0.f);
}
__device__ __forceinline__ float cons_max(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  cons_sync();
  if (lane == 0) red[w] = v;
  cons_sync();
  return warp_max(lane < kConsWarps ? red[lane] : -3.0e38f);
}

__device__ __forceinline__ unsigned long long am_key_m(float v, int idx) {
  const unsigned int hv = (unsigned int)float_to_ordered(v) ^ 0x80000000u;
  return ((unsigned long long)hv << 32) | (unsigned int)(0xFFFFFFFFu - (unsigned int)idx);
}

struct Smem {
  unsigned char* ring;
  uint64_t* full;
  uint64_t* empty;
  float* xs;         // staged f32 vector [kpad]
  int8_t* xq;        // quantised vector [kpad]
  float* part;       // [kTileRows][kMaxNkc] chunk partials
  float* rowv;       // [kTileRows] row values of a block (SwiGLU pairing)
  float* att;        // attention scratch (aliases xs / xq)
};

// Attention work items per kv head for this step: at least 48 positions per item (one CTA
// streams K/V at only ~20 GB/s through its ring while the machine prefetches weights, so a
// head is spread over many CTAs), at most as many items as CTAs allow; the last split of a
// head to finish merges the others.
__device__ __forceinline__ int att_splits(const MegaArgs& a, int pos) {
  return max(1, min(a.p.splits, (pos + 1 + 47) / 48));
}

__device__ __forceinline__ int rows_of(const MegaArgs& a, int type) {
  return max(0, min(a.p.N[type] - (int)blockIdx.x * a.p.rpc[type], a.p.rpc[type]));
}

// Stages the input vector of a matvec: src (f32) or the bf16 embedding row `erow`, RMS-
// normalised with `norm` when set; int8 mode quantises it. Returns the activation scale.
__device__ float stage_vec(const MegaArgs& a, const Smem& S, const float* src, const uint16_t* erow, float* x_out,
                           const float* norm, int K, int kpad, float* red) {
  const int tid = threadIdx.x;
  float ss = 0.f;
  for (int i = tid * 4; i < K; i += kCons * 4) {
    float4 v;
    if (erow) {
      const uint2 u = *reinterpret_cast<const uint2*>(erow + i);
      v = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                      __uint_as_float(u.y & 0xFFFF0000u));
      if (x_out) *reinterpret_cast<float4*>(x_out + i) = v;
    } else {
      v = __ldcg(reinterpret_cast<const float4*>(src + i));  // written by other CTAs: bypass L1
    }
    *reinterpret_cast<float4*>(S.xs + i) = v;
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  for (int i = K + tid; i < kpad; i += kCons) {
    S.xs[i] = 0.f;
    S.xq[i] = 0;
  }
  cons_sync();
  if (norm) {
    const float tot = cons_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
    for (int i = tid; i < K; i += kCons) S.xs[i] = __fmul_rn(__fmul_rn(S.xs[i], inv), norm[i]);
  }
  float xscale = 1.0f;
  if (a.int8) {
    float mx = 0.f;
    for (int i = tid; i < K; i += kCons) mx = fmaxf(mx, fabsf(S.xs[i]));
    mx = cons_max(mx, red);
    xscale = mx > 0.f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    const float qinv = __fdiv_rn(127.0f, fmaxf(mx, 1e-10f));
    for (int i = tid; i < K; i += kCons) {
      const float r = roundf(__fmul_rn(S.xs[i], qinv));
      S.xq[i] = (int8_t)fminf(fmaxf(r, -127.f), 127.f);
    }
  }
  cons_sync();
  return xscale;
}

enum { E_STORE = 0, E_RESID = 1, E_SWIGLU = 2, E_ARGMAX = 3 };

// Consumes this CTA's tiles of one matrix (blocks of R <= 32 rows, 512-byte chunks in
// order). Warp w owns rows 2w and 2w+1 of every block and accumulates them across the
// chunks in registers (each lane its 16 bytes of every chunk); one warp reduction per row,
// then lane 0 applies the epilogue: E_STORE out[row] = v; E_RESID out[row] += v; E_SWIGLU
// out[row / 2] = silu(v_gate) * v_up for its row pair (2j, 2j+1); E_ARGMAX folds (v, row)
// into `best` (and records the logit when requested). No CTA-wide synchronisation.
template <int EPI>
__device__ void run_matvec(const MegaArgs& a, const Smem& S, int type, int layer, float xscale, uint32_t& t,
                           volatile int* s_abort, float* out, unsigned long long& best) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = rows_of(a, type), R = a.p.R[type], nkc = a.p.nkc[type], ns = a.p.nslots;
  const int row0 = blockIdx.x * a.p.rpc[type];
  const float* ws = a.int8 ? a.wscale[type == T_LM ? a.L * 4 : layer * 4 + type] : nullptr;
  const int ra = 2 * warp, rb = 2 * warp + 1;  // rows of this warp inside a block
  for (int b0 = 0; b0 < rows; b0 += R) {
    const bool has_a = ra < R && b0 + ra < rows, has_b = rb < R && b0 + rb < rows;
    int ia = 0, ib = 0;
    float fa = 0.f, fb = 0.f;
    float old_a = 0.f, old_b = 0.f;  // residual rows, loaded while the tiles stream
    if (EPI == E_RESID && lane == 0) {
      if (has_a) old_a = __ldcg(out + row0 + b0 + ra);
      if (has_b) old_b = __ldcg(out + row0 + b0 + rb);
    }
    for (int kc = 0; kc < nkc; ++kc, ++t) {
      const int s = (int)(t % (uint32_t)ns);
      warp_ring_wait(a, &S.full[s], (t / (uint32_t)ns) & 1u, s_abort, 31);
      const unsigned char* tile = S.ring + (size_t)s * kSlot + lane * 16;
      if (a.int8) {
        const int4 xv = *reinterpret_cast<const int4*>(S.xq + kc * kChunkB + lane * 16);
        if (has_a) {
          const int4 w = *reinterpret_cast<const int4*>(tile + (size_t)ra * kChunkB);
          ia = __dp4a(w.x, xv.x, ia);
          ia = __dp4a(w.y, xv.y, ia);
          ia = __dp4a(w.z, xv.z, ia);
          ia = __dp4a(w.w, xv.w, ia);
        }
        if (has_b) {
          const int4 w = *reinterpret_cast<const int4*>(tile + (size_t)rb * kChunkB);
          ib = __dp4a(w.x, xv.x, ib);
          ib = __dp4a(w.y, xv.y, ib);
          ib = __dp4a(w.z, xv.z, ib);
          ib = __dp4a(w.w, xv.w, ib);
        }
      } else {
        const float* xb = S.xs + kc * (kChunkB / 2) + lane * 8;
        const float4 x0 = *reinterpret_cast<const float4*>(xb);
        const float4 x1 = *reinterpret_cast<const float4*>(xb + 4);
        float f[8];
        if (has_a) {
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(tile + (size_t)ra * kChunkB), f);
          fa = fmaf(f[0], x0.x, fa); fa = fmaf(f[1], x0.y, fa); fa = fmaf(f[2], x0.z, fa); fa = fmaf(f[3], x0.w, fa);
          fa = fmaf(f[4], x1.x, fa); fa = fmaf(f[5], x1.y, fa); fa = fmaf(f[6], x1.z, fa); fa = fmaf(f[7], x1.w, fa);
        }
        if (has_b) {
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(tile + (size_t)rb * kChunkB), f);
          fb = fmaf(f[0], x0.x, fb); fb = fmaf(f[1], x0.y, fb); fb = fmaf(f[2], x0.z, fb); fb = fmaf(f[3], x0.w, fb);
          fb = fmaf(f[4], x1.x, fb); fb = fmaf(f[5], x1.y, fb); fb = fmaf(f[6], x1.z, fb); fb = fmaf(f[7], x1.w, fb);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[s]);
    }
    if (!has_a) continue;  // warp-uniform
    float va, vb = 0.f;
    const int row_a = row0 + b0 + ra, row_b = row_a + 1;
    if (a.int8) {
      const int sa = warp_sum_i(ia), sb = warp_sum_i(ib);
      va = __fmul_rn(__fmul_rn((float)sa, xscale), ws[row_a]);
      if (has_b) vb = __fmul_rn(__fmul_rn((float)sb, xscale), ws[row_b]);
    } else {
      va = warp_sum(fa);
      vb = warp_sum(fb);
    }
    if (lane == 0) {
      if (EPI == E_SWIGLU) {
        if (has_b) out[row_a / 2] = silu_mul(va, vb);  // row_a is even
      } else if (EPI == E_STORE) {
        out[row_a] = va;
        if (has_b) out[row_b] = vb;
      } else if (EPI == E_RESID) {
        out[row_a] = __fadd_rn(va, old_a);
        if (has_b) out[row_b] = __fadd_rn(vb, old_b);
      } else {
        if (a.logits) {
          a.logits[row_a] = va;
          if (has_b) a.logits[row_b] = vb;
        }
        unsigned long long k = am_key_m(va, row_a);
        best = k > best ? k : best;
        if (has_b) {
          k = am_key_m(vb, row_b);
          best = k > best ? k : best;
        }
      }
    }
  }
}

// Attention work item (kv head, split) of one layer; see the file comment.
__device__ void run_attention(const MegaArgs& a, const Smem& S, int layer, int pos, uint32_t& t,
                              volatile int* s_abort, int* s_flag) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KVH = a.KVH, G = a.QH / a.KVH, splits = att_splits(a, pos), ns = a.p.nslots;
  const int item = blockIdx.x;
  if (item >= KVH * splits) return;
  const int kvh = item / splits, split = item % splits;
  const int total = pos + 1, chunk = (total + splits - 1) / splits;
  const int j0 = split * chunk, j1 = min(total, j0 + chunk);
  const int npre = max(0, min(j1, pos) - j0);
  const int qd = a.QH * kHdM, kvd = KVH * kHdM;
  float* raw = S.att;                          // [G + 2][128]: q heads, k, v
  float* hn = raw + (kMaxGq + 2) * kHdM;       // [G + 1][128] normalised q heads, k
  float* hr = hn + (kMaxGq + 1) * kHdM;        // [G + 1][128] rotated
  float* wm = hr + (kMaxGq + 1) * kHdM;        // [16][kMaxGq]
  float* wl = wm + kConsWarps * kMaxGq;        // [16][kMaxGq]
  float* wo = wl + kConsWarps * kMaxGq;        // [16][kMaxGq][128]
  const float* qn = a.lnorm[layer * 4 + 2];
  const float* kn = a.lnorm[layer * 4 + 3];
  for (int e = tid; e < (G + 2) * kHdM; e += kCons) {
    const int vec = e / kHdM, d = e % kHdM;
    const int row = vec < G ? (kvh * G + vec) * kHdM + d
                            : (vec == G ? qd + kvh * kHdM + d : qd + kvd + kvh * kHdM + d);
    raw[vec * kHdM + d] = __ldcg(a.qkv + row);
  }
  cons_sync();
  if (warp <= G) {  // q heads 0..G-1 and k (vec G): RMSNorm over 128 dims (kernels/mod.rs:1214-1240)
    const float4 v = *reinterpret_cast<const float4*>(raw + warp * kHdM + lane * 4);
    float s = v.x * v.x;
    s = fmaf(v.y, v.y, s);
    s = fmaf(v.z, v.z, s);
    s = fmaf(v.w, v.w, s);
    const float tot = warp_sum(s);
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)kHdM), a.eps)));
    const float* w = warp < G ? qn : kn;
    const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = lane * 4 + i;
      hn[warp * kHdM + d] = __fmul_rn(__fmul_rn(f[i], inv), w[d]);
    }
  }
  cons_sync();
  // NeoX rotation (generic path, kernels/mod.rs:1780-1788): pairs (d, d + 64)
  for (int e = tid; e < (G + 1) * kHdM; e += kCons) {
    const int vec = e / kHdM, d = e % kHdM;
    const float c = a.rope_cos[(size_t)pos * (kHdM / 2) + (d & 63)];
    const float sn = a.rope_sin[(size_t)pos * (kHdM / 2) + (d & 63)];
    const float nv = hn[vec * kHdM + d];
    hr[vec * kHdM + d] = d < kHdM / 2 ? __fadd_rn(__fmul_rn(nv, c), __fmul_rn(-hn[vec * kHdM + d + kHdM / 2], sn))
                                      : __fadd_rn(__fmul_rn(nv, c), __fmul_rn(hn[vec * kHdM + d - kHdM / 2], sn));
  }
  cons_sync();
  float* kb = a.k_cache + ((size_t)layer * KVH + kvh) * a.max_seq * kHdM;
  float* vb = a.v_cache + ((size_t)layer * KVH + kvh) * a.max_seq * kHdM;
  if (j0 <= pos && pos < j1) {  // this item's chunk holds the new position: append K/V
    if (tid < kHdM) kb[(size_t)pos * kHdM + tid] = hr[G * kHdM + tid];
    else if (tid < 2 * kHdM) vb[(size_t)pos * kHdM + tid - kHdM] = raw[(G + 1) * kHdM + tid - kHdM];
  }
  const float scale = 1.0f / sqrtf((float)kHdM);
  float m[kMaxGq], l[kMaxGq], o[kMaxGq][4];
#pragma unroll
  for (int g = 0; g < kMaxGq; ++g) {
    m[g] = -3.0e38f;
    l[g] = 0.f;
    o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
  }
  auto visit = [&](const float* krow, const float* vrow) {
    const float4 kv = *reinterpret_cast<const float4*>(krow + lane * 4);
    const float4 vv = *reinterpret_cast<const float4*>(vrow + lane * 4);
#pragma unroll
    for (int g = 0; g < kMaxGq; ++g) {
      if (g >= G) break;
      const float4 q = *reinterpret_cast<const float4*>(hr + g * kHdM + lane * 4);
      float p = q.x * kv.x;
      p = fmaf(q.y, kv.y, p);
      p = fmaf(q.z, kv.z, p);
      p = fmaf(q.w, kv.w, p);
      const float sc = __fmul_rn(warp_sum(p), scale);
      const float mn = fmaxf(m[g], sc);
      const float corr = expf(__fsub_rn(m[g], mn));
      const float e = expf(__fsub_rn(sc, mn));
      l[g] = fmaf(l[g], corr, e);
      o[g][0] = fmaf(o[g][0], corr, e * vv.x);
      o[g][1] = fmaf(o[g][1], corr, e * vv.y);
      o[g][2] = fmaf(o[g][2], corr, e * vv.z);
      o[g][3] = fmaf(o[g][3], corr, e * vv.w);
      m[g] = mn;
    }
  };
  for (int r0 = 0; r0 < npre; r0 += kKvRows, ++t) {
    const int s = (int)(t % (uint32_t)ns);
    warp_ring_wait(a, &S.full[s], (t / (uint32_t)ns) & 1u, s_abort, 32);
    const float* ks = reinterpret_cast<const float*>(S.ring + (size_t)s * kSlot);
    const float* vs = ks + kKvRows * kHdM;
    const int n = min(kKvRows, npre - r0);
    if (warp < n) visit(ks + warp * kHdM, vs + warp * kHdM);
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
  }
  if (j0 <= pos && pos < j1 && warp == (npre % kConsWarps)) visit(hr + G * kHdM, raw + (G + 1) * kHdM);
#pragma unroll
  for (int g = 0; g < kMaxGq; ++g) {
    if (g >= G) break;
    if (lane == 0) {
      wm[warp * kMaxGq + g] = m[g];
      wl[warp * kMaxGq + g] = l[g];
    }
    *reinterpret_cast<float4*>(wo + (warp * kMaxGq + g) * kHdM + lane * 4) =
        make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
  }
  cons_sync();
  if (splits == 1) {  // the whole head in this CTA: finish here
    for (int e = tid; e < G * kHdM; e += kCons) {
      const int g = e / kHdM, d = e % kHdM;
      float M = -3.0e38f;
      for (int w = 0; w < kConsWarps; ++w)
        if (wl[w * kMaxGq + g] > 0.f) M = fmaxf(M, wm[w * kMaxGq + g]);
      float L = 0.f, O = 0.f;
      for (int w = 0; w < kConsWarps; ++w) {
        const float lw = wl[w * kMaxGq + g];
        if (lw > 0.f) {
          const float f = expf(__fsub_rn(wm[w * kMaxGq + g], M));
          L = fmaf(lw, f, L);
          O = fmaf(wo[(w * kMaxGq + g) * kHdM + d], f, O);
        }
      }
      a.attn[(kvh * G + g) * kHdM + d] = __fdiv_rn(O, L);
    }
    return;
  }
  float* mypart = a.apart + ((size_t)(kvh * splits + split) * kMaxGq) * kApart;
  for (int e = tid; e < G * kHdM; e += kCons) {
    const int g = e / kHdM, d = e % kHdM;
    float M = -3.0e38f;
    for (int w = 0; w < kConsWarps; ++w)
      if (wl[w * kMaxGq + g] > 0.f) M = fmaxf(M, wm[w * kMaxGq + g]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kConsWarps; ++w) {
      const float lw = wl[w * kMaxGq + g];
      if (lw > 0.f) {
        const float f = expf(__fsub_rn(wm[w * kMaxGq + g], M));
        L = fmaf(lw, f, L);
        O = fmaf(wo[(w * kMaxGq + g) * kHdM + d], f, O);
      }
    }
    mypart[g * kApart + d] = O;
    if (d == 0) {
      mypart[g * kApart + kHdM] = M;
      mypart[g * kApart + kHdM + 1] = L;
    }
  }
  __threadfence();
  cons_sync();
  if (tid == 0) *s_flag = (atomicAdd(a.head_ticket + kvh, 1u) == (unsigned)splits - 1u);
  cons_sync();
  if (!*s_flag) return;
  __threadfence();
  // last split of this kv head: merge the splits into the attention output
  for (int e = tid; e < G * kHdM; e += kCons) {
    const int g = e / kHdM, d = e % kHdM;
    const float* pb = a.apart + ((size_t)kvh * splits * kMaxGq + g) * kApart;
    float M = -3.0e38f;
    for (int sp = 0; sp < splits; ++sp) {
      const float* q = pb + (size_t)sp * kMaxGq * kApart;
      if (__ldcg(q + kHdM + 1) > 0.f) M = fmaxf(M, __ldcg(q + kHdM));
    }
    float L = 0.f, O = 0.f;
    for (int sp = 0; sp < splits; ++sp) {
      const float* q = pb + (size_t)sp * kMaxGq * kApart;
      const float ls = __ldcg(q + kHdM + 1);
      if (ls > 0.f) {
        const float f = expf(__fsub_rn(__ldcg(q + kHdM), M));
        L = fmaf(ls, f, L);
        O = fmaf(__ldcg(q + d), f, O);
      }
    }
    a.attn[(kvh * G + g) * kHdM + d] = __fdiv_rn(O, L);
  }
  if (tid == 0) a.head_ticket[kvh] = 0u;
}

__global__ void __launch_bounds__(kThr, 1) decode_mega_kernel(const __grid_constant__ MegaArgs a) {
  extern __shared__ unsigned char sm_raw[];
  __shared__ float red[32];
  __shared__ int s_pos, s_step, s_tok, s_forced, s_flag;
  __shared__ volatile int s_abort;
  __shared__ unsigned long long s_best[kConsWarps];
  unsigned char* base = (unsigned char*)(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
  const MegaPlan& P = a.p;
  Smem S;
  S.ring = base;
  S.full = reinterpret_cast<uint64_t*>(base + (size_t)P.nslots * kSlot);
  S.empty = S.full + P.nslots;
  S.part = reinterpret_cast<float*>(S.empty + P.nslots);
  S.rowv = S.part + kTileRows * kMaxNkc;
  S.xs = S.rowv + kTileRows;
  S.xq = reinterpret_cast<int8_t*>(S.xs + P.kpad);
  S.att = S.xs;  // the attention phase stages nothing else
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < P.nslots; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], kConsWarps);
    }
    fence_mbar_init();
    const StepState st = *a.st;
    s_pos = st.pos;
    s_step = st.step;
    s_tok = st.cur_token;
    s_forced = st.forced_mode;
    s_abort = (int)ld_acquire(a.gbar + 2);
  }
  __syncthreads();
  const int pos = s_pos;

  if (warp == kConsWarps) {
    // ---- producer: every tile of the step, in consumption order
    if (lane == 0) {
      const int ns = P.nslots;
      uint32_t t = 0;
      bool ok = true;
      auto acquire = [&]() -> int {
        const int s = (int)(t % (uint32_t)ns);
        if (t >= (uint32_t)ns && !ring_wait(a, &S.empty[s], ((t / (uint32_t)ns) - 1u) & 1u, &s_abort, 33)) return -1;
        return s;
      };
      auto issue_rows = [&](int type, int layer) {
        const CUtensorMap* map = a.maps + (type == T_LM ? a.L * 4 : layer * 4 + type);
        const int rows = rows_of(a, type), R = P.R[type], nkc = P.nkc[type];
        const int row0 = blockIdx.x * P.rpc[type];
        for (int b0 = 0; b0 < rows && ok; b0 += R)
          for (int kc = 0; kc < nkc && ok; ++kc) {
            const int s = acquire();
            if (s < 0) {
              ok = false;
              break;
            }
            mbar_expect_tx(&S.full[s], (uint32_t)(R * kChunkB));
            tma_tile(S.ring + (size_t)s * kSlot, map, kc * (kChunkB / 2), row0 + b0, &S.full[s]);
            ++t;
          }
      };
      const int KVH = a.KVH, splits = att_splits(a, pos), item = blockIdx.x;
      const int total = pos + 1, chunk = (total + splits - 1) / splits;
      for (int l = 0; l < a.L && ok; ++l) {
        issue_rows(T_QKV, l);
        if (item < KVH * splits) {
          const int kvh = item / splits, split = item % splits;
          const int j0 = split * chunk, j1 = min(total, j0 + chunk), npre = max(0, min(j1, pos) - j0);
          const float* kb = a.k_cache + ((size_t)l * KVH + kvh) * a.max_seq * kHdM;
          const float* vb = a.v_cache + ((size_t)l * KVH + kvh) * a.max_seq * kHdM;
          for (int r0 = 0; r0 < npre && ok; r0 += kKvRows) {
            const int s = acquire();
            if (s < 0) {
              ok = false;
              break;
            }
            const int n = min(kKvRows, npre - r0);
            const uint32_t bytes = (uint32_t)(n * kHdM * 4);
            unsigned char* dst = S.ring + (size_t)s * kSlot;
            mbar_expect_tx(&S.full[s], 2 * bytes);
            bulk_g2s(dst, kb + (size_t)(j0 + r0) * kHdM, bytes, &S.full[s]);
            bulk_g2s(dst + kKvRows * kHdM * 4, vb + (size_t)(j0 + r0) * kHdM, bytes, &S.full[s]);
            ++t;
          }
        }
        issue_rows(T_O, l);
        issue_rows(T_GU, l);
        issue_rows(T_DOWN, l);
      }
      if (ok) issue_rows(T_LM, 0);
    }
    return;
  }

  // ---- consumers
  uint32_t t = 0;
  unsigned long long best = 0ull;
  const int H = a.H, qd = a.QH * kHdM;
  for (int l = 0; l < a.L; ++l) {
    MegaTimeline ph;
    {  // QKV projection (input RMSNorm fused; layer 0 takes its input from the embedding)
      ph.open(a, 10);
      const uint16_t* erow = nullptr;
      if (l == 0 && s_tok >= 0) erow = reinterpret_cast<const uint16_t*>(a.embed) + (size_t)s_tok * H;
      const float xs = stage_vec(a, S, a.x, erow, (erow && blockIdx.x == 0) ? a.x : nullptr, a.lnorm[l * 4], H,
                                 P.kpad, red);
      ph.mark(2);
      run_matvec<E_STORE>(a, S, T_QKV, l, xs, t, &s_abort, a.qkv, best);
      ph.mark(3);
    }
    grid_sync(a, &s_abort, 41);
    ph.open(a, 11);
    run_attention(a, S, l, pos, t, &s_abort, &s_flag);
    ph.mark(3);
    grid_sync(a, &s_abort, 42);
    {  // O projection + residual
      ph.open(a, 12);
      const float xs = stage_vec(a, S, a.attn, nullptr, nullptr, nullptr, qd, P.kpad, red);
      ph.mark(2);
      run_matvec<E_RESID>(a, S, T_O, l, xs, t, &s_abort, a.x, best);
      ph.mark(3);
    }
    grid_sync(a, &s_abort, 43);
    {  // gate/up (post-attention RMSNorm fused) + SwiGLU
      ph.open(a, 13);
      const float xs = stage_vec(a, S, a.x, nullptr, nullptr, a.lnorm[l * 4 + 1], H, P.kpad, red);
      ph.mark(2);
      run_matvec<E_SWIGLU>(a, S, T_GU, l, xs, t, &s_abort, a.ffn, best);
      ph.mark(3);
    }
    grid_sync(a, &s_abort, 44);
    {  // down projection + residual
      ph.open(a, 14);
      const float xs = stage_vec(a, S, a.ffn, nullptr, nullptr, nullptr, a.I, P.kpad, red);
      ph.mark(2);
      run_matvec<E_RESID>(a, S, T_DOWN, l, xs, t, &s_abort, a.x, best);
      ph.mark(3);
    }
    grid_sync(a, &s_abort, 45);
  }
  {  // lm_head (final RMSNorm fused) + greedy argmax
    MegaTimeline ph;
    ph.open(a, 15);
    const float xs = stage_vec(a, S, a.x, nullptr, nullptr, a.final_norm, H, P.kpad, red);
    ph.mark(2);
    run_matvec<E_ARGMAX>(a, S, T_LM, 0, xs, t, &s_abort, nullptr, best);
    ph.mark(3);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t2 = __shfl_xor_sync(0xffffffffu, best, o);
    best = t2 > best ? t2 : best;
  }
  if (lane == 0) s_best[warp] = best;
  cons_sync();
  if (tid == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kConsWarps; ++w) b = s_best[w] > b ? s_best[w] : b;
    a.am_part[blockIdx.x] = b;
    __threadfence();
    s_flag = (atomicAdd(a.am_ticket, 1u) == gridDim.x - 1u);
  }
  cons_sync();
  if (s_flag && warp == 0) {
    __threadfence();
    unsigned long long b = 0ull;
    for (int i = lane; i < (int)gridDim.x; i += 32) {
      const unsigned long long u = __ldcg(a.am_part + i);
      b = u > b ? u : b;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t2 = __shfl_xor_sync(0xffffffffu, b, o);
      b = t2 > b ? t2 : b;
    }
    if (lane == 0) {
      const int tok = (int)(0xFFFFFFFFu - (unsigned int)(b & 0xFFFFFFFFull));
      const int step = s_step;
      a.tokens[step] = tok;
      StepState* st = a.st;
      st->cur_token = (s_forced && a.forced) ? a.forced[step] : tok;
      st->step = step + 1;
      st->pos = pos + 1;
      *a.am_ticket = 0u;
    }
  }
}

}  // namespace
}  // namespace qasr

namespace qasr {

struct MegaState {
  MegaArgs args{};            // constant part (weights, plan, scratch)
  unsigned long long* bar_last = nullptr;
  int grid = 0;
  bool int8 = false;
  std::vector<void*> allocs;
  ~MegaState() {
    for (void* p : allocs) cudaFree(p);
  }
  template <typename T>
  T* alloc(size_t n) {
    void* p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) return nullptr;
    allocs.push_back(p);
    return (T*)p;
  }
};

namespace {
constexpr int kMegaSmemBudget = 225 * 1024;

bool plan_mega(const DecodeArgs& a, int grid, MegaPlan& p) {
  const int esz = a.int8 ? 1 : 2;
  const int qd = a.q_heads * kHdM, kvd = a.kv_heads * kHdM;
  const int N[5] = {qd + 2 * kvd, a.hidden, 2 * a.inter, a.hidden, a.vocab};
  const int K[5] = {a.hidden, qd, a.hidden, a.inter, a.hidden};
  int kpad = 0;
  for (int t = 0; t < 5; ++t) {
    p.N[t] = N[t];
    p.K[t] = K[t];
    int rpc = (N[t] + grid - 1) / grid;
    if (t == T_GU) rpc += rpc & 1;
    const int nblk = (rpc + kTileRows - 1) / kTileRows;
    int R = (rpc + nblk - 1) / nblk;
    if (t == T_GU) R = 2 * ((rpc + 2 * nblk - 1) / (2 * nblk));
    p.rpc[t] = rpc;
    p.R[t] = R;
    p.nkc[t] = (K[t] * esz + kChunkB - 1) / kChunkB;
    if (R > kTileRows || p.nkc[t] > kMaxNkc || K[t] % 4 != 0 || (K[t] * esz) % 16 != 0) return false;
    kpad = std::max(kpad, p.nkc[t] * kChunkB / esz);
  }
  if (a.q_heads % a.kv_heads != 0 || a.q_heads / a.kv_heads > kMaxGq || a.kv_heads > grid) return false;
  p.splits = grid / a.kv_heads;
  p.kpad = kpad;
  const size_t att = ((kMaxGq + 2) * kHdM + 2 * (kMaxGq + 1) * kHdM + 2 * kConsWarps * kMaxGq +
                      kConsWarps * kMaxGq * kHdM) * sizeof(float);
  const size_t region = std::max<size_t>((size_t)kpad * 5, att);
  const size_t rest = 1024 + (size_t)(kTileRows * kMaxNkc + kTileRows) * 4 + region;
  const int nslots = (int)std::min<size_t>(12, (kMegaSmemBudget - rest) / (kSlot + 16));
  if (nslots < 4) return false;
  p.nslots = nslots;
  p.smem = (int)(rest + (size_t)nslots * (kSlot + 16));
  return true;
}
}  // namespace

MegaState* mega_create(const DecodeArgs& a) {
  int dev = 0, nsm = 0, coop = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (!coop || nsm <= 0) return nullptr;
  MegaPlan p{};
  if (!plan_mega(a, nsm, p)) return nullptr;
  if (cudaFuncSetAttribute(decode_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel, kThr, p.smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    return nullptr;
  }
  auto* m = new MegaState();
  m->grid = nsm;
  m->int8 = a.int8;
  MegaArgs& g = m->args;
  g.H = a.hidden; g.QH = a.q_heads; g.KVH = a.kv_heads; g.I = a.inter; g.V = a.vocab; g.L = a.layers;
  g.eps = a.eps; g.int8 = a.int8 ? 1 : 0; g.p = p;
  g.final_norm = a.final_norm; g.embed = a.embed; g.rope_cos = a.rope_cos; g.rope_sin = a.rope_sin;
  // tensor maps (one per weight matrix) and per-layer pointer tables, in device memory
  const int nm = a.layers * 4 + 1;
  std::vector<CUtensorMap> maps(nm);
  std::vector<const float*> ws(nm, nullptr), ln((size_t)a.layers * 4, nullptr);
  const int esz = a.int8 ? 1 : 2;
  bool ok = true;
  for (int l = 0; l < a.layers && ok; ++l) {
    const void* W[4] = {a.w_qkv[l], a.w_o[l], a.w_gu[l], a.w_down[l]};
    const float* S4[4] = {a.s_qkv[l], a.s_o[l], a.s_gu[l], a.s_down[l]};
    for (int t = 0; t < 4 && ok; ++t) {
      ok = make_tma_2d_u16(&maps[l * 4 + t], W[t], p.N[t], p.K[t] * esz / 2, kChunkB / 2, p.R[t]);
      ws[l * 4 + t] = S4[t];
    }
    ln[l * 4] = a.n1[l];
    ln[l * 4 + 1] = a.n2[l];
    ln[l * 4 + 2] = a.qn[l];
    ln[l * 4 + 3] = a.kn[l];
  }
  if (ok) ok = make_tma_2d_u16(&maps[nm - 1], a.lm_w, p.N[T_LM], p.K[T_LM] * esz / 2, kChunkB / 2, p.R[T_LM]);
  ws[nm - 1] = a.lm_s;
  CUtensorMap* dmaps = m->alloc<CUtensorMap>(nm);
  const float** dws = m->alloc<const float*>(nm);
  const float** dln = m->alloc<const float*>((size_t)a.layers * 4);
  float* apart = m->alloc<float>((size_t)a.kv_heads * p.splits * kMaxGq * kApart);
  unsigned* tickets = m->alloc<unsigned>((size_t)a.kv_heads + 1 + 3);
  unsigned long long* am_part = m->alloc<unsigned long long>(nsm);
  m->bar_last = m->alloc<unsigned long long>(64);
  if (!ok || !dmaps || !dws || !dln || !apart || !tickets || !am_part ||
      cudaMemcpy(dmaps, maps.data(), nm * sizeof(CUtensorMap), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(dws, ws.data(), nm * sizeof(float*), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(dln, ln.data(), ln.size() * sizeof(float*), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(tickets, 0, ((size_t)a.kv_heads + 4) * sizeof(unsigned)) != cudaSuccess) {
    delete m;
    return nullptr;
  }
  g.maps = dmaps;
  g.wscale = dws;
  g.lnorm = dln;
  g.apart = apart;
  g.head_ticket = tickets;
  g.am_ticket = tickets + a.kv_heads;
  g.gbar = tickets + a.kv_heads + 1;
  g.am_part = am_part;
  return m;
}

void mega_destroy(MegaState* m) { delete m; }

bool mega_reset(MegaState* m, cudaStream_t s) {
  return cudaMemsetAsync(m->args.head_ticket, 0, ((size_t)m->args.KVH + 4) * sizeof(unsigned), s) == cudaSuccess;
}

bool mega_step(MegaState* m, const DecodeArgs& a, cudaStream_t s) {
  MegaArgs g = m->args;
  g.k_cache = a.k_cache;
  g.v_cache = a.v_cache;
  g.max_seq = a.max_seq;
  g.x = a.x;
  g.qkv = a.qkv;
  g.attn = a.attn;
  g.ffn = a.ffn;
  g.st = a.st;
  g.tokens = a.tokens;
  g.forced = a.forced;
  g.logits = a.logits;
  g.err = a.err;
  g.tl = a.tl;
  g.tl_count = a.tl_count;
  g.bar_last = m->bar_last;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->grid);
  cfg.blockDim = dim3(kThr);
  cfg.dynamicSmemBytes = g.p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_mega_kernel, g) == cudaSuccess;
}

}  // namespace qasr
