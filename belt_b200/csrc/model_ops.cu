// The element-wise steps of a compressed layer's attention block around the backend (plugins/vllm_lrkv/vllm_lrkv/
// models/qwen3_5_latent.py:204-217):
//   * q_norm_rope: the query half of each head's q_gate_proj output -> zero-centred RMSNorm (weight 1 + w, fp32) and
//     the partial NeoX rotation of its first `rot` channels at the token's position (BF16 cos / sin table), one BF16
//     rounding at the end (the query side of ``fused_qk_rmsnorm_rope_gate``, :209-212, with no key heads);
//   * gate_mul: attn_out * sigmoid(gate), the gate being the second half of each head's q_gate_proj output (:215).
// One warp per (token, head) for the norm (8 channels per lane, 16-byte loads, shuffle reductions, the rotation
// partner rot / 16 lanes away); 8 channels per thread for the gate.
#include "common.cuh"
#include "launch.h"

namespace belt {

__global__ void __launch_bounds__(256) q_norm_rope_kernel(const QNormRopeParams p) {
  const int warp_global = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (warp_global >= p.T * p.H) return;
  const int t = warp_global / p.H, h = warp_global - t * p.H;
  const __nv_bfloat16* src = p.qg + static_cast<long long>(t) * p.qg_st + static_cast<long long>(h) * p.qg_sh;
  const uint4 raw = *reinterpret_cast<const uint4*>(src + 8 * lane);
  const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
  float x[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w4[i] << 16);
    x[2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / 256.f + p.eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = x[i] * inv * (1.f + p.w[8 * lane + i]);
  // NeoX rotation of channels [0, rot): channel c < rot / 2 pairs with c + rot / 2, rot / 16 lanes away
  const int half_lanes = p.rot >> 4;
  const bool rotated = 8 * lane < p.rot;
  const bool first = 8 * lane < (p.rot >> 1);
  float partner[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float up = __shfl_down_sync(0xffffffffu, x[i], half_lanes);   // lane + half_lanes
    const float dn = __shfl_up_sync(0xffffffffu, x[i], half_lanes);     // lane - half_lanes
    partner[i] = first ? up : dn;
  }
  if (rotated) {
    long long pos = p.pos_i64 ? static_cast<const long long*>(p.positions)[t]
                              : static_cast<long long>(static_cast<const int32_t*>(p.positions)[t]);
    pos = pos < 0 ? 0 : (pos >= p.max_pos ? p.max_pos - 1 : pos);
    const __nv_bfloat16* cs = p.cos_sin + pos * p.rot;
    const int c0 = first ? 8 * lane : 8 * lane - (p.rot >> 1);   // index of the pair's frequency
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float cv = __bfloat162float(cs[c0 + i]), sv = __bfloat162float(cs[(p.rot >> 1) + c0 + i]);
      x[i] = first ? x[i] * cv - partner[i] * sv : x[i] * cv + partner[i] * sv;
    }
  }
  __nv_bfloat16* dst = p.q + static_cast<long long>(t) * p.q_st + static_cast<long long>(h) * p.q_sh;
  *reinterpret_cast<uint4*>(dst + 8 * lane) =
      make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
}

__global__ void __launch_bounds__(256) gate_mul_kernel(const GateMulParams p) {
  const long long i = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;   // 8-channel unit
  const long long units = static_cast<long long>(p.T) * p.H * 32;
  if (i >= units) return;
  const int u = static_cast<int>(i & 31);
  const long long th = i >> 5;
  const int t = static_cast<int>(th / p.H), h = static_cast<int>(th - static_cast<long long>(t) * p.H);
  const uint4 a = *reinterpret_cast<const uint4*>(p.attn + t * p.attn_st + h * p.attn_sh + 8 * u);
  const uint4 g = *reinterpret_cast<const uint4*>(p.gate + t * p.gate_st + h * p.gate_sh + 8 * u);
  const uint32_t av[4] = {a.x, a.y, a.z, a.w}, gv[4] = {g.x, g.y, g.z, g.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float a0 = __uint_as_float(av[k] << 16), a1 = __uint_as_float(av[k] & 0xFFFF0000u);
    const float g0 = __uint_as_float(gv[k] << 16), g1 = __uint_as_float(gv[k] & 0xFFFF0000u);
    o[k] = pack_bf16(a0 / (1.f + __expf(-g0)), a1 / (1.f + __expf(-g1)));
  }
  *reinterpret_cast<uint4*>(p.out + t * p.out_st + h * p.out_sh + 8 * u) = make_uint4(o[0], o[1], o[2], o[3]);
}

cudaError_t launch_q_norm_rope(const QNormRopeParams& p, cudaStream_t stream) {
  const long long warps = static_cast<long long>(p.T) * p.H;
  if (warps == 0) return cudaSuccess;
  q_norm_rope_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gate_mul(const GateMulParams& p, cudaStream_t stream) {
  const long long units = static_cast<long long>(p.T) * p.H * 32;
  if (units == 0) return cudaSuccess;
  gate_mul_kernel<<<static_cast<unsigned>((units + 255) / 256), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace belt
