// FP32 SIMT GEMM with fused epilogues: C = epi(A[M][K] * B[N][K]^T).
// This is the exact-f32 path (same arithmetic class as the reference's cblas_sgemm) and
// the fallback-free reference point for the tensor-core GEMM's parity tests.
#include "common.h"
#include "kernels.h"
#include "dev_util.cuh"

namespace qasr {

namespace {
constexpr int BM = 128, BN = 128, BK = 16, TM = 8, TN = 8;

template <bool BF32>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmArgs a) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tx = tid % 16, ty = tid / 16;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < a.K; k0 += BK) {
    // A tile: 128 rows x 16 cols = 512 float4, 2 per thread.
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      int idx = tid + r * 256;
      int row = idx / 4, c4 = (idx % 4) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m0 + row < a.M) v = *reinterpret_cast<const float4*>(a.A + (size_t)(m0 + row) * a.lda + k0 + c4);
      As[c4 + 0][row] = v.x;
      As[c4 + 1][row] = v.y;
      As[c4 + 2][row] = v.z;
      As[c4 + 3][row] = v.w;
    }
    if (BF32) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        int idx = tid + r * 256;
        int row = idx / 4, c4 = (idx % 4) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n0 + row < a.N)
          v = *reinterpret_cast<const float4*>((const float*)a.B + (size_t)(n0 + row) * a.ldb + k0 + c4);
        Bs[c4 + 0][row] = v.x;
        Bs[c4 + 1][row] = v.y;
        Bs[c4 + 2][row] = v.z;
        Bs[c4 + 3][row] = v.w;
      }
    } else {
      int row = tid / 2, c8 = (tid % 2) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (n0 + row < a.N)
        v = *reinterpret_cast<const uint4*>((const __nv_bfloat16*)a.B + (size_t)(n0 + row) * a.ldb + k0 + c8);
      float f[8];
      bf16x8_to_f32(v, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) Bs[c8 + j][row] = f[j];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float av[TM], bv[TN];
      float4 a0 = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[k][64 + ty * 4]);
      float4 b0 = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
      float4 b1 = *reinterpret_cast<const float4*>(&Bs[k][64 + tx * 4]);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
      av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
      bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }

  // Epilogue. Thread rows: ty*4+{0..3}, 64+ty*4+{0..3}; cols: tx*4+{0..3}, 64+tx*4+{0..3}.
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= a.M) continue;
#pragma unroll
    for (int jh = 0; jh < 2; ++jh) {
      int nb = n0 + jh * 64 + tx * 4;
      if (a.epi == EPI_SWIGLU) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          int n = nb + 2 * p;
          if (n + 1 < a.N) a.C[(size_t)m * a.ldc + n / 2] = silu_mul(acc[i][jh * 4 + 2 * p], acc[i][jh * 4 + 2 * p + 1]);
        }
        continue;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int n = nb + j;
        if (n >= a.N) continue;
        float v = acc[i][jh * 4 + j];
        a.C[(size_t)m * a.ldc + n] = apply_epi(a, m, n, v);
      }
    }
  }
}
}  // namespace

void gemm_simt(const GemmArgs& a, cudaStream_t s) {
  dim3 grid(ceil_div(a.N, BN), ceil_div(a.M, BM));
  if (a.b_is_f32) gemm_simt_kernel<true><<<grid, 256, 0, s>>>(a);
  else gemm_simt_kernel<false><<<grid, 256, 0, s>>>(a);
}

}  // namespace qasr
