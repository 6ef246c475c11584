// Log-sum-exp fold of one chunk's attention result into the running result, in place: the step of the reference's
// chunked prefill that merges every context chunk into the output with vLLM's merge_attn_states
// (plugins/vllm_lrkv/vllm_lrkv/latent_backend.py:300-320):
//     m = max(lse, plse), wo = e^(lse - m), wc = e^(plse - m)
//     out = bf16((out wo + part wc) / (wo + wc)),  lse = m + log(wo + wc)
// A part row whose LSE is -inf (a query that saw none of the chunk's keys) leaves its row unchanged; a running row with
// LSE -inf takes the part row. Rows come from a piece table (destination row, source row, count per piece).
// One warp per (row, head), 8 warps per CTA (grid: rows x 3 head groups); a lane owns 8 channels (one 16-byte load of
// each operand).
#include "common.cuh"
#include "launch.h"

namespace belt {

__global__ void __launch_bounds__(256) attn_fold_kernel(const __grid_constant__ AttnFoldParams p) {
  const int r = blockIdx.x;
  int pi = 0;
  while (pi + 1 < p.num_pieces && r >= p.piece_row0[pi + 1]) ++pi;
  const long long i = r - p.piece_row0[pi];
  const long long dst = p.piece_dst[pi] + i, src = p.piece_src[pi] + i;
  const int h = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (h >= p.H) return;
  float* lse = p.lse + dst * p.lse_st + h;
  const float lo = *lse, lc = p.plse[src * p.plse_st + h];
  if (lc == -INFINITY) return;
  uint4* o = reinterpret_cast<uint4*>(p.out + dst * p.out_st + static_cast<long long>(h) * p.out_sh) + lane;
  const uint4 c = reinterpret_cast<const uint4*>(p.part + src * p.part_st + static_cast<long long>(h) * p.part_sh)[lane];
  if (lo == -INFINITY) {
    *o = c;
    __syncwarp();
    if (lane == 0) *lse = lc;
    return;
  }
  const float m = fmaxf(lo, lc);
  const float wo = __expf(lo - m), wc = __expf(lc - m);
  const float inv = 1.f / (wo + wc);
  const uint4 a = *o;
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
  uint32_t rw[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float a0 = __uint_as_float(aw[k] << 16), a1 = __uint_as_float(aw[k] & 0xFFFF0000u);
    const float c0 = __uint_as_float(cw[k] << 16), c1 = __uint_as_float(cw[k] & 0xFFFF0000u);
    rw[k] = pack_bf16((a0 * wo + c0 * wc) * inv, (a1 * wo + c1 * wc) * inv);
  }
  *o = make_uint4(rw[0], rw[1], rw[2], rw[3]);
  __syncwarp();
  if (lane == 0) *lse = m + __logf(wo + wc);
}

cudaError_t launch_attn_fold(const AttnFoldParams& p, cudaStream_t stream) {
  const int rows = p.piece_row0[p.num_pieces];
  if (rows == 0) return cudaSuccess;
  attn_fold_kernel<<<dim3(rows, (p.H + 7) / 8), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace belt
