// Latent cache write: the new tokens' rows into their paged slots, the reference's ``_latent_rows``
// (plugins/vllm_lrkv/vllm_lrkv/latent_ops.py:85-135):
//     per token t and KV group g:  k_pre = U_g c_g (BF16 operands, FP32 accumulation, all 256 channels)
//                                  row[cols_g] = bf16(c_g * rsqrt(mean(k_pre^2) + eps))
//     row[lk : W] = c[lk : W] (V latent and alignment gaps, unscaled); slot < 0 (padding) is skipped.
// Block (x, g): 16 tokens of group g (g < G) or the V-part copy (g == G). For a group, 256 threads = 256 channels;
// the 16 tokens' latent coordinates sit in shared memory and every U_g row is read once per block.
// belt_latent_rows_to_cache uses this kernel only for layouts the fused write's c-input mode (proj_write.cu) does not
// take: a group spread over more than five 64-column chunks, or a u_cat that is not 16-byte aligned.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int kTok = 16;
constexpr int kMaxRank = 256;
}

__device__ __forceinline__ long long load_slot(const CacheWriteParams& p, int t) {
  return p.slots_i64 ? static_cast<const long long*>(p.slots)[t] : static_cast<long long>(static_cast<const int32_t*>(p.slots)[t]);
}

__global__ void __launch_bounds__(256) cache_write_kernel(const CacheWriteParams p) {
  __shared__ float cs[kTok][kMaxRank];
  __shared__ float red[8][kTok];
  __shared__ float inv_s[kTok];
  __shared__ long long slot_s[kTok];
  const int g = blockIdx.y;
  const int tok0 = blockIdx.x * kTok;
  const int tid = threadIdx.x;
  if (tid < kTok) {
    const int t = tok0 + tid;
    long long s = t < p.T ? load_slot(p, t) : -1;
    if (s >= p.num_slots) s = -1;   // beyond the cache: treated as padding
    slot_s[tid] = s;
  }
  __syncthreads();
  if (g == p.G) {
    // V latent and gaps: columns [lk, W)
    const int width = p.W - p.lk;
    for (int i = tid; i < kTok * width; i += 256) {
      const int tk = i / width, col = p.lk + i % width;
      const long long s = slot_s[tk];
      if (s < 0) continue;
      p.cache[(s / p.page) * p.sblk + (s % p.page) * p.stok + col] = p.c[(tok0 + tk) * p.sct + col];
    }
    return;
  }
  const int a_lo = p.a_lo[g], a_n = p.a_n[g], b_lo = p.b_lo[g];
  const int r = a_n + p.b_n[g];
  for (int i = tid; i < kTok * r; i += 256) {
    const int tk = i / r, k = i % r;
    const int col = k < a_n ? a_lo + k : b_lo + k - a_n;
    const int t = tok0 + tk;
    cs[tk][k] = t < p.T ? __bfloat162float(p.c[t * p.sct + col]) : 0.f;
  }
  __syncthreads();
  // k_pre for channel d = tid of every token
  float acc[kTok] = {};
  const int ld = p.G * kD;
  for (int k = 0; k < r; ++k) {
    const int col = k < a_n ? a_lo + k : b_lo + k - a_n;
    const float u = __bfloat162float(p.u_cat[static_cast<long long>(col) * ld + g * kD + tid]);
#pragma unroll
    for (int tk = 0; tk < kTok; ++tk) acc[tk] = fmaf(cs[tk][k], u, acc[tk]);
  }
  const int lane = tid & 31, w = tid >> 5;
#pragma unroll
  for (int tk = 0; tk < kTok; ++tk) {
    float v = acc[tk] * acc[tk];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[w][tk] = v;
  }
  __syncthreads();
  if (tid < kTok) {
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sq += red[i][tid];
    inv_s[tid] = rsqrtf(sq / kD + p.eps);
  }
  __syncthreads();
  for (int i = tid; i < kTok * r; i += 256) {
    const int tk = i / r, k = i % r;
    const long long s = slot_s[tk];
    if (s < 0) continue;
    const int col = k < a_n ? a_lo + k : b_lo + k - a_n;
    p.cache[(s / p.page) * p.sblk + (s % p.page) * p.stok + col] = __float2bfloat16_rn(cs[tk][k] * inv_s[tk]);
  }
}

cudaError_t launch_cache_write(const CacheWriteParams& p, cudaStream_t stream) {
  if (p.T == 0) return cudaSuccess;
  dim3 grid((p.T + kTok - 1) / kTok, p.G + 1);
  cache_write_kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace belt
