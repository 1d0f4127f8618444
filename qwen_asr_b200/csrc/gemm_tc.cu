// Tensor-core GEMM for sm_100a: C = epi(A[M][K] * B[N][K]^T) on tcgen05 with the
// accumulator in TMEM, operands moved by TMA (cp.async.bulk.tensor, no multicast).
//
// Precision: B holds bf16 weights (exact: the reference upcasts the same bf16 values to
// f32). A holds f32 activations; it is split into bf16 hi + lo parts (a = hi + lo up to
// 2^-16 relative) and both are multiplied against B into the same f32 accumulator, which
// keeps the contraction at f32-level accuracy, as the reference's sgemm is.
//
// Tile 128 x 128 x 64 per CTA, 4-stage smem ring. 128 threads: thread 0 issues TMA,
// thread 32 issues MMAs, then all four warps drain TMEM (warp w owns rows 32w..32w+31).
#include <cuda.h>

#include <mutex>

#include "bulk.cuh"
#include "common.h"
#include "dev_util.cuh"
#include "kernels.h"

namespace qasr {
namespace {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 4;
constexpr int kTileA = BM * BK * 2;  // 16 KB (bf16)
constexpr int kTileB = BN * BK * 2;  // 16 KB
constexpr int kStage = 2 * kTileA + kTileB;
constexpr int kSmem = STAGES * kStage + 1024 /*align*/ + 256 /*barriers*/;

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

// Instruction descriptor, kind::f16: f32 accumulator, bf16 A and B, both K-major.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accum));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define TMEM_LD32(taddr, r)                                                                                       \
  asm volatile(                                                                                                   \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                              \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),           \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),     \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),   \
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])    \
      : "r"(taddr))

__global__ void __launch_bounds__(128, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap map_ahi,
                                                         const __grid_constant__ CUtensorMap map_alo,
                                                         const __grid_constant__ CUtensorMap map_b, GemmArgs a,
                                                         int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStage);
  uint64_t* empty = full + STAGES;
  uint64_t* accum_bar = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nk = (a.K + BK - 1) / BK;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {  // TMEM: 128 f32 columns = the 128 x 128 accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    // ---- TMA producer
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES) mbar_wait(&empty[s], (uint32_t)((kt / STAGES) - 1) & 1u, err, 11);
      unsigned char* st = smem + s * kStage;
      mbar_expect_tx(&full[s], kStage);
      tma_load_2d(st, &map_ahi, kt * BK, m0, &full[s]);
      tma_load_2d(st + kTileA, &map_alo, kt * BK, m0, &full[s]);
      tma_load_2d(st + 2 * kTileA, &map_b, kt * BK, n0, &full[s]);
    }
  } else if (tid == 32) {
    // ---- MMA issuer
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % STAGES;
      mbar_wait(&full[s], (uint32_t)(kt / STAGES) & 1u, err, 12);
      asm volatile("tcgen05.fence::after_thread_sync;");
      const uint32_t sa = smem_u32(smem + s * kStage);
      const uint32_t sal = sa + kTileA, sb = sa + 2 * kTileA;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {  // K = 16 per instruction = 32 bytes along the row
        const uint64_t bd = sw128_desc(sb + kk * 32);
        mma_bf16(tmem, sw128_desc(sa + kk * 32), bd, (kt > 0 || kk > 0) ? 1u : 0u);
        mma_bf16(tmem, sw128_desc(sal + kk * 32), bd, 1u);
      }
      mma_commit(&empty[s]);  // stage reusable once these MMAs have read it
    }
    mma_commit(accum_bar);
  }
  __syncwarp();

  // ---- epilogue: TMEM -> registers -> fused epilogue -> global
  mbar_wait(accum_bar, 0, err, 13);
  asm volatile("tcgen05.fence::after_thread_sync;");
  const int m = m0 + warp * 32 + lane;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    uint32_t r[32];
    TMEM_LD32(trow + c0, r);
    asm volatile("tcgen05.wait::ld.sync.aligned;");
    if (m >= a.M) continue;
    const int nb = n0 + c0;
    if (a.epi == EPI_SWIGLU) {
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        if (nb + j + 1 < a.N)
          a.C[(size_t)m * a.ldc + (nb + j) / 2] = silu_mul(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (nb + j < a.N) a.C[(size_t)m * a.ldc + nb + j] = apply_epi(a, m, nb + j, __uint_as_float(r[j]));
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
}

// a -> (hi, lo) bf16 with a = hi + lo to 2^-16 relative; rows [M][K] packed (ld = K).
__global__ void split_bf16_kernel(const float* __restrict__ A, int lda, int M, int K, __nv_bfloat16* __restrict__ hi,
                                  __nv_bfloat16* __restrict__ lo) {
  const long total = (long)M * (K / 4);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / (K / 4)), c = (int)(i % (K / 4)) * 4;
    float4 v = *reinterpret_cast<const float4*>(A + (size_t)r * lda + c);
    float f[4] = {v.x, v.y, v.z, v.w};
    __nv_bfloat16 h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = __float2bfloat16_rn(f[j]);
      l[j] = __float2bfloat16_rn(__fsub_rn(f[j], __bfloat162float(h[j])));
    }
    *reinterpret_cast<uint2*>(hi + (size_t)r * K + c) = *reinterpret_cast<uint2*>(h);
    *reinterpret_cast<uint2*>(lo + (size_t)r * K + c) = *reinterpret_cast<uint2*>(l);
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

// Row-major bf16 [rows][cols] (ld elements), box = box_rows x 64, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int rows, int cols, int ld, int box_rows) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct TcScratch {
  __nv_bfloat16* hi = nullptr;
  __nv_bfloat16* lo = nullptr;
  size_t cap = 0;
  int* err = nullptr;
};
TcScratch g_tc[16];
std::mutex g_tc_mu;

}  // namespace

bool gemm_tc_available() { return get_encode() != nullptr; }

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

bool gemm_tc(const GemmArgs& a, cudaStream_t s) {
  if (a.b_is_f32 || a.K % 16 != 0 || (a.ldb * 2) % 16 != 0) return false;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 16) return false;
  TcScratch& sc = g_tc[dev];
  {
    std::lock_guard<std::mutex> lk(g_tc_mu);
    size_t need = (size_t)a.M * a.K;
    if (sc.cap < need) {
      // Grow-only split buffers (the engine calls this outside any stream capture).
      cudaStreamSynchronize(s);
      if (sc.hi) cudaFree(sc.hi);
      if (sc.lo) cudaFree(sc.lo);
      size_t cap = std::max(need, (size_t)1 << 22);
      if (cudaMalloc(&sc.hi, cap * 2) != cudaSuccess || cudaMalloc(&sc.lo, cap * 2) != cudaSuccess) {
        sc.hi = sc.lo = nullptr;
        sc.cap = 0;
        return false;
      }
      sc.cap = cap;
    }
    if (!sc.err) {
      if (cudaMalloc(&sc.err, sizeof(int)) != cudaSuccess) return false;
      cudaMemset(sc.err, 0, sizeof(int));
      cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    }
  }
  const long total = (long)a.M * (a.K / 4);
  split_bf16_kernel<<<(int)std::min<long>((total + 255) / 256, 148L * 16), 256, 0, s>>>(a.A, a.lda, a.M, a.K, sc.hi,
                                                                                       sc.lo);
  CUtensorMap mh, ml, mb;
  if (!make_map(&mh, sc.hi, a.M, a.K, a.K, BM) || !make_map(&ml, sc.lo, a.M, a.K, a.K, BM) ||
      !make_map(&mb, a.B, a.N, a.K, a.ldb, BN))
    return false;
  dim3 grid(ceil_div(a.N, BN), ceil_div(a.M, BM));
  gemm_tc_kernel<<<grid, 128, kSmem, s>>>(mh, ml, mb, a, sc.err);
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
