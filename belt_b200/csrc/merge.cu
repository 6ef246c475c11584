// LSE merge of every request's split-KV segments, the reference's ``_merge_segments``
// (plugins/vllm_lrkv/vllm_lrkv/cute_decode.py:681-722):
//     a[b, h, :] = sum_s exp(lse_s - m) part[s, h, :lv] / sum_s exp(lse_s - m),   lse[b, h] = m + log(sum)
// over the segments seg_base[b] .. seg_base[b + 1] - 1; a request without segments (padding) gets zeros and -inf.
// One CTA per (request, head); the segment weights go through shared memory in blocks of 256.
#include "common.cuh"
#include "launch.h"

namespace belt {

__global__ void __launch_bounds__(128) merge_kernel(const MergeParams p) {
  __shared__ float wts[256];
  __shared__ float red[4];
  __shared__ float m_s, den_s;
  const int b = blockIdx.x, h = blockIdx.y;
  const int s0 = p.seg_base[b];
  const int n = p.seg_base[b + 1] - s0;
  const float* base = p.part + static_cast<long long>(s0) * p.ps + h * p.ph;
  // max of the segment LSEs
  float m = -INFINITY;
  for (int s = threadIdx.x; s < n; s += 128) m = fmaxf(m, base[static_cast<long long>(s) * p.ps + p.lv]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) m_s = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  m = m_s;
  float den = 0.f;
  for (int s = threadIdx.x; s < n; s += 128) den += __expf(base[static_cast<long long>(s) * p.ps + p.lv] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = den;
  __syncthreads();
  if (threadIdx.x == 0) den_s = red[0] + red[1] + red[2] + red[3];
  __syncthreads();
  den = den_s;
  const bool has = den > 0.f;
  const float inv = has ? 1.f / den : 0.f;
  constexpr int kPer = 8;   // features per thread per pass (lv <= 128 * 8)
  for (int f0 = 0; f0 < p.lv; f0 += 128 * kPer) {
    float acc[kPer] = {};
    for (int s0w = 0; s0w < n; s0w += 256) {
      const int cnt = min(256, n - s0w);
      __syncthreads();
      for (int i = threadIdx.x; i < cnt; i += 128)
        wts[i] = __expf(base[static_cast<long long>(s0w + i) * p.ps + p.lv] - m);
      __syncthreads();
      for (int i = 0; i < cnt; ++i) {
        const float w = wts[i];
        const float* row = base + static_cast<long long>(s0w + i) * p.ps;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int f = f0 + k * 128 + threadIdx.x;
          if (f < p.lv) acc[k] = fmaf(w, row[f], acc[k]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int f = f0 + k * 128 + threadIdx.x;
      if (f < p.lv) p.out[b * p.sob + h * p.soh + f] = __float2bfloat16_rn(acc[k] * inv);
    }
  }
  if (threadIdx.x == 0) p.lse[b * p.slb + h] = has ? m + __logf(den) : -INFINITY;
}

cudaError_t launch_merge(const MergeParams& p, cudaStream_t stream) {
  if (p.num_reqs == 0) return cudaSuccess;
  merge_kernel<<<dim3(p.num_reqs, p.nh), 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace belt
