// Grouped GEMM over KV groups, the operation of the reference's ``_group_gemm``
// (plugins/vllm_lrkv/vllm_lrkv/latent_ops.py:23-44): for the rows r = t * hpg + j of group g,
//     Out[t, g * hpg + j, n] = X[t, g * hpg + j, :] @ W[g, :, n]      (BF16 operands, FP32 accumulation, BF16 out)
// It serves both
//   * block_diag_query (latent_ops.py:67-73): X = the normed rotated query [T, H, 256], W = qmap [G, 256, KQ]; only
//     the columns where the group's map is non-zero (its latent columns and its RoPE chunk, passed as column runs)
//     are computed, the others are written as zeros;
//   * up_project (latent_ops.py:76-81): X = the merged latent output [T, H, r_v], W = U_v^T [G, r_v, 256].
// Tiles of 64 rows x 64 columns, 32-deep K steps through shared memory, 256 threads with 4 x 4 outputs each.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int BM = 64, BN = 64, BK = 32;
}

__global__ void __launch_bounds__(256) group_gemm_kernel(const GroupGemmParams p) {
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int g = blockIdx.z;
  const int r0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int rows = p.T * p.hpg;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

  // does this column tile hold any computed column of group g?
  bool any = false;
  for (int i = 0; i < p.nruns[g]; ++i) any |= p.run_lo[g][i] < n0 + BN && p.run_hi[g][i] > n0;

  float acc[4][4] = {};
  if (any) {
    for (int k0 = 0; k0 < p.K; k0 += BK) {
      for (int i = tid; i < BM * BK; i += 256) {
        const int rr = i / BK, kk = i % BK;
        const int r = r0 + rr, k = k0 + kk;
        float v = 0.f;
        if (r < rows && k < p.K) {
          const int t = r / p.hpg, h = g * p.hpg + r % p.hpg;
          v = __bfloat162float(p.X[t * p.sxt + h * p.sxh + k]);
        }
        xs[kk][rr] = v;
      }
      for (int i = tid; i < BK * BN; i += 256) {
        const int kk = i / BN, nn = i % BN;
        const int k = k0 + kk, n = n0 + nn;
        float v = 0.f;
        if (k < p.K && n < p.N) v = __bfloat162float(p.W[g * p.swg + k * p.swk + n * p.swn]);
        ws[kk][nn] = v;
      }
      __syncthreads();
#pragma unroll 8
      for (int kk = 0; kk < BK; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i] = xs[kk][ty * 4 + i];
          b[i] = ws[kk][tx * 4 + i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= rows) continue;
    const int t = r / p.hpg, h = g * p.hpg + r % p.hpg;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= p.N) continue;
      bool live = false;
      for (int q = 0; q < p.nruns[g]; ++q) live |= n >= p.run_lo[g][q] && n < p.run_hi[g][q];
      p.Out[t * p.sot + h * p.soh + n] = __float2bfloat16_rn(live ? acc[i][j] : 0.f);
    }
  }
}

cudaError_t launch_group_gemm(const GroupGemmParams& p, cudaStream_t stream) {
  const int rows = p.T * p.hpg;
  dim3 grid((rows + BM - 1) / BM, (p.N + BN - 1) / BN, p.G);
  if (rows == 0) return cudaSuccess;
  group_gemm_kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace belt
