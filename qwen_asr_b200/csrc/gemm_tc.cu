// Tensor-core GEMM for sm_100a: C = epi(A[M][K] * B[N][K]^T) on tcgen05 with the
// accumulators in TMEM and every operand moved by TMA (cp.async.bulk.tensor; each CTA loads its own tiles).
//
// Precision. B holds bf16 weights, exact (the reference upcasts the same bf16 values to
// f32 before its sgemm). A holds f32 activations and enters as three bf16 planes,
// a = hi + mid + lo, each plane the bf16 rounding of what the planes before it left over,
// so the three carry all 24 significand bits of an f32 (exact except for rare
// sub-2^-126 remainders). Every product of a bf16 plane with a bf16 weight is exact in the
// f32 accumulator, so the contraction has the f32 accumulation error of an sgemm, not the
// 2^-9 or 2^-17 representation error of one or two bf16 terms. The planes come either from
// the producing kernel (LayerNorm/RMSNorm, GEMM epilogues, attention) or from split3_kernel.
//
// Schedule. A persistent grid (one CTA per SM) walks work units (m tile, n tile, k split)
// in a fixed order. Tiles are 128 x BN, BN = 128 for wide outputs and 64 for narrow ones.
// Warp 0 issues TMA into a 3-stage ring (per stage the three A planes and the B tile), warp 1
// issues 12 MMAs (128 x BN x 16) per stage into one of two TMEM accumulators, and warps 2-9
// drain the other accumulator (two warps per TMEM lane quarter, each half the columns):
// tcgen05.ld, a transpose through shared memory, then the fused epilogue with coalesced
// row-wise stores. So the epilogue of one unit overlaps the mainloop of the next.
//
// Split K. A GEMM with few output tiles splits K into S parts so that about 148 CTAs work.
// S depends only on the call's (N, K) and its split policy, never on M, so a row's result
// never depends on how many other rows share the call (batched segments and streams equal
// single ones bit for bit). Each split stores its f32 partial tile to a workspace; the last
// split of a tile to arrive (ticket) sums the S partials in split order and applies the
// epilogue, so the sum order is fixed too.
#include <cuda.h>

#include <mutex>
#include <unordered_map>

#include "bulk.cuh"
#include "common.h"
#include "dev_util.cuh"
#include "kernels.h"

namespace qasr {
namespace {

constexpr int BM = 128, BK = 64, STAGES = 3, NPART = 3;
constexpr int kTile = BM * BK * 2;  // 16 KB: one bf16 A plane tile
constexpr int kEpiWarps = 8;
constexpr int kEpiPitch = 33;       // floats per staged row (bank-conflict padding)
constexpr int kEpiBytes = kEpiWarps * 32 * kEpiPitch * 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;
template <int BN>
struct Tile {
  static constexpr int kB = BN * BK * 2;              // B tile bytes
  static constexpr int kStage = NPART * kTile + kB;   // 56 or 64 KB
  static constexpr int kSmem = 1024 + STAGES * kStage + kEpiBytes + 256;
  // kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both K-major, M = 128
  static constexpr uint32_t kIdesc =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};
constexpr int kSms = 148;
constexpr int kMaxSplit = 16;

struct TcParams {
  int M, N, K, MT, NT, S, nk, units;
  int epi;
  float* C;
  int ldc;
  const float* bias;
  const float* resid;
  int ldr;
  __nv_bfloat16* cs;  // optional split-plane output [3][plane] of rows of cs_ld
  int cs_ld;
  long long cs_plane;
  float* ws;     // split-K partial tiles [tile][S][BM][BN]
  int* tickets;  // [tile], zero at rest
  int* err;
  // Optional timeline (debug): per CTA 8 %globaltimer stamps: entry, set-up done, first stage
  // landed, first unit's MMAs committed, first unit's accumulator ready, first unit stored,
  // (unused), exit.
  unsigned long long* tl;
};

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused with 128B swizzle, K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;            // version
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

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

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

#define TMEM_LD32(taddr, r)                                                                                       \
  asm volatile(                                                                                                   \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                              \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),           \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),     \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),   \
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])    \
      : "r"(taddr))

__device__ __forceinline__ void unit_coords(const TcParams& p, int u, int& mt, int& nt, int& s) {
  mt = u % p.MT;
  const int t = u / p.MT;
  s = t % p.S;
  nt = t / p.S;
}
__device__ __forceinline__ void split_range(const TcParams& p, int s, int& k0, int& k1) {
  k0 = (int)((long)s * p.nk / p.S);
  k1 = (int)((long)(s + 1) * p.nk / p.S);
}

// Final value of one output element (or SwiGLU pair) to C and/or the split planes.
__device__ __forceinline__ void store_out(const TcParams& p, int m, int n, float v) {
  if (p.C) p.C[(size_t)m * p.ldc + n] = v;
  if (p.cs) {
    __nv_bfloat16 h, md, l;
    split3_bf16(v, h, md, l);
    __nv_bfloat16* q = p.cs + (size_t)m * p.cs_ld + n;
    q[0] = h;
    q[p.cs_plane] = md;
    q[2 * p.cs_plane] = l;
  }
}
// One 32x32 block (rows m0.., columns n0..) staged in st[32][kEpiPitch]: epilogue + stores,
// lane = column, so every store instruction writes consecutive addresses of one row. All
// global loads of the block (bias, residual rows) are issued before the first use.
__device__ __forceinline__ void epilogue_block(const TcParams& p, const float* st, int m0, int n0, int lane) {
  if (p.epi == EPI_SWIGLU) {
    // columns (2j, 2j+1) = (gate, up) -> output column n/2 + j; two rows per pass
#pragma unroll 4
    for (int rr = 0; rr < 32; rr += 2) {
      const int r = rr + (lane >> 4), j = lane & 15, m = m0 + r, n = n0 + 2 * j;
      if (m < p.M && n + 1 < p.N) store_out(p, m, n >> 1, silu_mul(st[r * kEpiPitch + 2 * j], st[r * kEpiPitch + 2 * j + 1]));
    }
    return;
  }
  const int n = n0 + lane;
  const bool n_ok = n < p.N;
  const float bias = (p.bias && n_ok && p.epi != EPI_STORE) ? p.bias[n] : 0.f;
  float res[32];
  if (p.epi == EPI_RESID) {
#pragma unroll
    for (int r = 0; r < 32; ++r) res[r] = (n_ok && m0 + r < p.M) ? p.resid[(size_t)(m0 + r) * p.ldr + n] : 0.f;
  }
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    const int m = m0 + r;
    if (m >= p.M || !n_ok) continue;
    const float acc = st[r * kEpiPitch + lane];
    float v;
    switch (p.epi) {
      case EPI_BIAS: v = __fadd_rn(acc, bias); break;
      case EPI_BIAS_GELU: v = gelu_tanh(__fadd_rn(acc, bias)); break;
      case EPI_RESID: v = __fadd_rn(acc, p.bias ? __fadd_rn(res[r], bias) : res[r]); break;
      default: v = acc;
    }
    store_out(p, m, n, v);
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                                                              const __grid_constant__ CUtensorMap map_b,
                                                              const TcParams p) {
  using T = Tile<BN>;
  constexpr int kChunks = BN / 64;  // 32-column chunks per epilogue warp (each warp: half the columns)
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* epi_st = reinterpret_cast<float*>(smem + STAGES * T::kStage);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * T::kStage + kEpiBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_flag = last_flag + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  unsigned long long* tl = (p.tl && blockIdx.x < kSms) ? p.tl + blockIdx.x * 8 : nullptr;
  if (tl && tid == 0) tl[0] = global_timer_ns();

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {  // TMEM: two 128 x BN f32 accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  if (tl && tid == 0) tl[1] = global_timer_ns();

  if (warp == 0) {
    // ---- TMA producer
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
        int mt, nt, s, k0, k1;
        unit_coords(p, u, mt, nt, s);
        split_range(p, s, k0, k1);
        for (int kt = k0; kt < k1; ++kt, ++it) {
          const int st = it % STAGES;
          if (it >= STAGES && !mbar_wait(&empty[st], (uint32_t)((it / STAGES) - 1) & 1u, p.err, 11)) {
            *abort_flag = 1;
            break;
          }
          unsigned char* sp = smem + st * T::kStage;
          mbar_expect_tx(&full[st], T::kStage);
#pragma unroll
          for (int q = 0; q < NPART; ++q) tma_load_3d(sp + q * kTile, &map_a, kt * BK, mt * BM, q, &full[st]);
          tma_load_2d(sp + NPART * kTile, &map_b, kt * BK, nt * BN, &full[st]);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      int it = 0, lt = 0;
      for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x, ++lt) {
        int mt, nt, s, k0, k1;
        unit_coords(p, u, mt, nt, s);
        split_range(p, s, k0, k1);
        const int ab = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[ab], (uint32_t)((lt >> 1) - 1) & 1u, p.err, 12)) {
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t acc = tmem + (uint32_t)(ab * BN);
        bool ok = true;
        for (int kt = k0; kt < k1; ++kt, ++it) {
          const int st = it % STAGES;
          if (!mbar_wait(&full[st], (uint32_t)(it / STAGES) & 1u, p.err, 13)) {
            ok = false;
            break;
          }
          if (tl && it == 0) tl[2] = global_timer_ns();
          asm volatile("tcgen05.fence::after_thread_sync;");
          const uint32_t sa = smem_u32(smem + st * T::kStage), sb = sa + NPART * kTile;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {  // K = 16 per instruction = 32 bytes along the row
            const uint64_t bd = sw128_desc(sb + kk * 32);
#pragma unroll
            for (int q = 0; q < NPART; ++q)
              mma_bf16(acc, sw128_desc(sa + q * kTile + kk * 32), bd, T::kIdesc,
                       (kt > k0 || kk > 0 || q > 0) ? 1u : 0u);
          }
          mma_commit(&empty[st]);  // stage reusable once these MMAs have read it
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mma_commit(&acc_full[ab]);
        if (tl && lt == 0) tl[3] = global_timer_ns();
      }
    }
  } else {
    // ---- epilogue warps 2..9: TMEM lane quarter q = warp % 4 -> tile rows 32q..32q+31;
    // column half h = (warp - 2) / 4 -> columns [h * BN / 2, (h + 1) * BN / 2)
    const int q = warp & 3, half = (warp - 2) >> 2;
    float* st = epi_st + (warp - 2) * 32 * kEpiPitch;
    int lt = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++lt) {
      int mt, nt, s;
      unit_coords(p, u, mt, nt, s);
      const int ab = lt & 1;
      if (!mbar_wait(&acc_full[ab], (uint32_t)(lt >> 1) & 1u, p.err, 14)) {
        *abort_flag = 1;
        break;
      }
      if (tl && tid == 64 && lt == 0) tl[4] = global_timer_ns();
      asm volatile("tcgen05.fence::after_thread_sync;");
      const int m0 = mt * BM + q * 32, nb = nt * BN + half * (BN / 2);
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN + half * (BN / 2));
      const int tile = nt * p.MT + mt;
      float* wsp = p.S > 1 ? p.ws + ((size_t)tile * p.S + s) * (BM * BN) : nullptr;
#pragma unroll 1
      for (int c = 0; c < kChunks; ++c) {
        uint32_t r[32];
        TMEM_LD32(trow + c * 32, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;");
#pragma unroll
        for (int j = 0; j < 32; ++j) st[lane * kEpiPitch + j] = __uint_as_float(r[j]);
        __syncwarp();
        if (wsp) {
          // raw partial: rows 32q.. of the tile, this warp's 32 columns
          float* w = wsp + (size_t)(q * 32) * BN + half * (BN / 2) + c * 32 + lane;
#pragma unroll 8
          for (int rr = 0; rr < 32; ++rr) w[(size_t)rr * BN] = st[rr * kEpiPitch + lane];
        } else {
          epilogue_block(p, st, m0, nb + c * 32, lane);
        }
        __syncwarp();
      }
      asm volatile("tcgen05.fence::before_thread_sync;");
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      if (wsp) {
        __threadfence();
        epi_bar();
        if (tid == 64) {
          const int t = atomicAdd(p.tickets + tile, 1);
          *last_flag = (t == p.S - 1);
        }
        epi_bar();
        if (*last_flag) {
          __threadfence();
          const float* w0 = p.ws + (size_t)tile * p.S * (BM * BN) + (size_t)(q * 32) * BN + half * (BN / 2) + lane;
#pragma unroll 1
          for (int c = 0; c < kChunks; ++c) {
            // partials summed in split order; two splits' 32 rows in flight per round
            float v[32];
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) v[rr] = __ldcg(w0 + (size_t)rr * BN + c * 32);
#pragma unroll 1
            for (int k = 1; k < p.S; k += 2) {
              const bool two = k + 1 < p.S;
              float t0[32], t1[32];
#pragma unroll
              for (int rr = 0; rr < 32; ++rr) {
                t0[rr] = __ldcg(w0 + (size_t)k * (BM * BN) + (size_t)rr * BN + c * 32);
                t1[rr] = two ? __ldcg(w0 + (size_t)(k + 1) * (BM * BN) + (size_t)rr * BN + c * 32) : 0.f;
              }
#pragma unroll
              for (int rr = 0; rr < 32; ++rr) {
                v[rr] = __fadd_rn(v[rr], t0[rr]);
                if (two) v[rr] = __fadd_rn(v[rr], t1[rr]);
              }
            }
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) st[rr * kEpiPitch + lane] = v[rr];
            __syncwarp();
            epilogue_block(p, st, m0, nb + c * 32, lane);
            __syncwarp();
          }
          epi_bar();
          if (tid == 64) p.tickets[tile] = 0;  // ready for the next call
        }
        epi_bar();
      }
      if (tl && tid == 64 && lt == 0) tl[5] = global_timer_ns();
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  if (tl && tid == 0) tl[7] = global_timer_ns();
}

// f32 rows [M][lda] -> bf16 planes hi/mid/lo [3][plane] of rows [M][K] (ld = K).
__global__ void split3_kernel(const float* __restrict__ A, int lda, int M, int K, __nv_bfloat16* __restrict__ out,
                              long long plane) {
  const long total = (long)M * (K / 4);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / (K / 4)), c = (int)(i % (K / 4)) * 4;
    const float4 v = *reinterpret_cast<const float4*>(A + (size_t)r * lda + c);
    const float f[4] = {v.x, v.y, v.z, v.w};
    __nv_bfloat16 h[4], m[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) split3_bf16(f[j], h[j], m[j], l[j]);
    __nv_bfloat16* o = out + (size_t)r * K + c;
    *reinterpret_cast<uint2*>(o) = *reinterpret_cast<uint2*>(h);
    *reinterpret_cast<uint2*>(o + plane) = *reinterpret_cast<uint2*>(m);
    *reinterpret_cast<uint2*>(o + 2 * plane) = *reinterpret_cast<uint2*>(l);
  }
}

// ---- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

// Tensor maps are encoded once per (base, shape) and reused: weights never move and the
// engine's activation buffers only change address when they grow.
struct MapKey {
  const void* base;
  long long rows, cols, ld, planes, plane, box_rows;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && ld == o.ld && planes == o.planes &&
           plane == o.plane && box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.base);
    for (long long v : {k.rows, k.cols, k.ld, k.planes, k.plane, k.box_rows})
      h = h * 1000003u ^ std::hash<long long>()(v);
    return h;
  }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// bf16 operand [planes][rows][cols] (row pitch ld, plane pitch `plane` elements), box =
// 64 columns x box_rows rows x 1 plane, 128-byte swizzle; out-of-range boxes read zeros.
bool operand_map(CUtensorMap* out, const void* base, int rows, int cols, int ld, int planes, long long plane,
                 int box_rows) {
  MapKey key{base, rows, cols, ld, planes, plane, box_rows};
  std::lock_guard<std::mutex> lk(g_map_mu);
  auto itm = g_maps.find(key);
  if (itm != g_maps.end()) {
    *out = itm->second;
    return true;
  }
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)plane * 2};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap m;
  if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, planes > 1 ? 3 : 2, const_cast<void*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return true;
}

struct TcScratch {
  __nv_bfloat16* planes = nullptr;  // split3 output
  size_t planes_cap = 0;
  float* ws = nullptr;
  size_t ws_cap = 0;
  int* tickets = nullptr;
  size_t tickets_cap = 0;
  int* err = nullptr;
  bool init = false;
};
TcScratch g_tc[16];
std::mutex g_tc_mu;
long g_fallbacks = 0;
unsigned long long* g_gemm_tl = nullptr;  // debug timeline target (qwen_asr_debug_gemm_timeline)

// Grow-only device buffer (the engine calls gemm outside stream capture).
template <typename T>
bool grow(T*& p, size_t& cap, size_t need, cudaStream_t s, bool zero) {
  if (cap >= need && p) return true;
  cudaStreamSynchronize(s);
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
  need = std::max(need, (size_t)4096);
  if (cudaMalloc(&p, need * sizeof(T)) != cudaSuccess) {
    p = nullptr;
    return false;
  }
  if (zero && cudaMemset(p, 0, need * sizeof(T)) != cudaSuccess) return false;
  cap = need;
  return true;
}

}  // namespace

bool gemm_tc_available() { return get_encode() != nullptr; }

void gemm_tc_set_timeline(unsigned long long* dev_buf) { g_gemm_tl = dev_buf; }

long gemm_tc_fallbacks() {
  std::lock_guard<std::mutex> lk(g_tc_mu);
  return g_fallbacks;
}
void gemm_tc_note_fallback() {
  std::lock_guard<std::mutex> lk(g_tc_mu);
  ++g_fallbacks;
}

// Output tile width: 128 columns when that already gives about half a wave of 128 x 128
// tiles for a ~384-row call, or when M alone fills the GPU (the conv stem: fewer column tiles
// mean fewer re-reads of the three A planes), else 64. The width never changes a result
// (each output element accumulates its own K sequence).
int gemm_tile_n(int N, int M) { return (M >= 2048 || 3 * ceil_div(N, 128) >= 74) ? 128 : 64; }

int gemm_split_k(int N, int K, int policy) {
  if (policy > 0) return std::min(policy, kMaxSplit);
  if (policy < 0) return 1;
  const int nk = ceil_div(K, BK), nt = ceil_div(N, gemm_tile_n(N, 384));
  // fill about one wave of 148 CTAs for a ~384-row call (3 row tiles), >= 8 k-steps per split
  const int s = std::min(kSms / (3 * nt), nk / 8);
  return std::max(1, std::min(s, kMaxSplit));
}

bool make_tma_2d_u16(void* map, const void* base, int rows, int cols, int box_cols, int box_rows, bool swizzle128) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc((CUtensorMap*)map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void split3_rows(const float* A, int lda, int M, int K, __nv_bfloat16* out, long long plane, cudaStream_t s) {
  const long total = (long)M * (K / 4);
  if (total <= 0) return;
  split3_kernel<<<(int)std::min<long>((total + 255) / 256, kSms * 16L), 256, 0, s>>>(A, lda, M, K, out, plane);
}

bool gemm_tc(const GemmArgs& a, cudaStream_t s) {
  if (a.b_is_f32 || a.K % 16 != 0 || (a.ldb * 2) % 16 != 0 || a.epi == EPI_LOG10_MAX) return false;
  if (!a.C && !a.c_split) return false;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 16) return false;
  TcScratch& sc = g_tc[dev];
  const int BN = gemm_tile_n(a.N, a.M);
  const int MT = ceil_div(a.M, BM), NT = ceil_div(a.N, BN), nk = ceil_div(a.K, BK);
  const int S = std::min(gemm_split_k(a.N, a.K, a.split_k), nk);
  const __nv_bfloat16* planes = a.a_split;
  int pld = a.a_split_ld;
  long long pplane = a.a_split_plane;
  {
    std::lock_guard<std::mutex> lk(g_tc_mu);
    if (!sc.init) {
      if (cudaMalloc(&sc.err, sizeof(int)) != cudaSuccess) return false;
      cudaMemset(sc.err, 0, sizeof(int));
      cudaFuncSetAttribute(gemm_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, Tile<64>::kSmem);
      cudaFuncSetAttribute(gemm_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, Tile<128>::kSmem);
      sc.init = true;
    }
    if (!planes) {
      if (!grow(sc.planes, sc.planes_cap, (size_t)3 * a.M * a.K, s, false)) return false;
    }
    if (S > 1) {
      if (!grow(sc.ws, sc.ws_cap, (size_t)MT * NT * S * BM * BN, s, false) ||
          !grow(sc.tickets, sc.tickets_cap, (size_t)MT * NT, s, true))
        return false;
    }
  }
  if (!planes) {
    pplane = (long long)a.M * a.K;
    pld = a.K;
    split3_rows(a.A, a.lda, a.M, a.K, sc.planes, pplane, s);
    planes = sc.planes;
  }
  if ((pld * 2) % 16 != 0 || (pplane * 2) % 16 != 0) return false;
  CUtensorMap ma, mb;
  if (!operand_map(&ma, planes, a.M, a.K, pld, NPART, pplane, BM) ||
      !operand_map(&mb, a.B, a.N, a.K, a.ldb, 1, 0, BN))
    return false;
  TcParams p;
  p.M = a.M; p.N = a.N; p.K = a.K; p.MT = MT; p.NT = NT; p.S = S; p.nk = nk; p.units = MT * NT * S;
  p.epi = a.epi; p.C = a.C; p.ldc = a.ldc; p.bias = a.bias; p.resid = a.resid; p.ldr = a.ldr;
  p.cs = a.c_split; p.cs_ld = a.c_split_ld; p.cs_plane = a.c_split_plane;
  p.ws = sc.ws; p.tickets = sc.tickets; p.err = sc.err; p.tl = g_gemm_tl;
  const int grid = std::min(p.units, kSms);
  if (BN == 128)
    gemm_tc_kernel<128><<<grid, kThreads, Tile<128>::kSmem, s>>>(ma, mb, p);
  else
    gemm_tc_kernel<64><<<grid, kThreads, Tile<64>::kSmem, s>>>(ma, mb, p);
  return true;
}

int gemm_tc_error() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 16 || !g_tc[dev].err) return 0;
  int e = 0;
  cudaMemcpy(&e, g_tc[dev].err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e) cudaMemset(g_tc[dev].err, 0, sizeof(int));
  return e;
}

}  // namespace qasr
