// Segment merge and V up-projection in one kernel: the reference's ``merge_segments`` (plugins/vllm_lrkv/vllm_lrkv/
// cute_decode.py:681-722) followed by ``up_project`` (latent_ops.py:76-81), with the merged latent output kept in
// shared memory instead of a [B, H, r_v] buffer:
//     a[b, h, :]   = bf16( sum_s exp(lse_s - m) part[s, h, :r_v] / sum_s exp(lse_s - m) )   over b's segments
//     lse[b, h]    = m + log(sum_s exp(lse_s - m))                 (-inf and a zero output for a request without any)
//     out[b, h, :] = bf16( U_v,g(h) a[b, h, :] )                   (FP32 accumulation)
// The roundings are the unfused path's (a rounded to BF16 before the projection), so the two agree to one BF16 ulp.
//
// One CTA per (head, tile of 32 requests), 1024 threads (a warp per request):
//   * thread 0 streams U_v^T of the head's group ([r_v, 256], channels contiguous) in 64-deep K blocks, four boxes of
//     64 channels x 64 k (MN-major, 128-byte swizzle) per stage, from the start (it does not depend on the merge);
//   * warp j merges request j: its lanes reduce the segment LSEs (a running max and sum per lane, then across the
//     warp) and write a as the K-major B operand (32 requests x r_v, 128-byte swizzle). With 16-byte aligned partial
//     rows (the backend pads their stride to a multiple of 4 floats) a lane owns 4 consecutive features per 128 and
//     loads them as float4, two segments' rows in flight at once, the first two issued together with the LSE loads;
//     otherwise the rows are swept with scalar loads, four segments in flight;
//   * thread 32 issues tcgen05 out^T[channel, request] += U_v^T[channel, k] a^T[k, request]: M = 128 channels (two
//     halves), N = 32 requests, K = 16 per instruction, into TMEM;
//   * epilogue (warps 0-3): thread (warp w, lane l) holds channel 32 w + l of both halves for the 32 requests; with an
//     aligned output it stages them as [request][256 channels] BF16 in the (consumed) first ring stage and every
//     thread of the CTA then stores 16 bytes (one request row = 512 contiguous bytes per warp); otherwise a warp's
//     stores of one request cover 32 consecutive channels (64 bytes).
// The U_v K blocks past the ring's first fill are prefetched into L2 at the start, so that their reloads after the
// merge come from L2.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int kMuThreads = 1024;
constexpr int kMuReqs = 32;                         // requests per CTA (the MMA's N)
constexpr int kMuStageBytes = 4 * 64 * 128;         // 256 channels x 64 k x 2 B = 32 KB
constexpr int kMuStages = 5;                        // 160 KB: five of the (at most ten) K blocks in flight
constexpr int kMuMaxChunks = 10;                    // r_v <= 640
constexpr int kMuBChunk = kMuReqs * 128;            // 32 requests x 64 k x 2 B = 4 KB per K block
constexpr int kMuOffB = kMuStages * kMuStageBytes;  // 160 KB
constexpr int kMuOffW = kMuOffB + kMuMaxChunks * kMuBChunk;   // per-warp segment weights
constexpr int kMuWeights = 64;                      // segment weights staged per pass, per warp (more than 32)
constexpr int kMuOffBars = kMuOffW + (kMuThreads / 32) * kMuWeights * 4;
// barriers: full[5], empty[5], done
constexpr int uFull = 0, uEmpty = kMuStages, uDone = 2 * kMuStages, kMuBars = 2 * kMuStages + 1;

// Offset of element (row, k) of a K-major 128-byte-swizzled operand of 64-column chunks of `rows` rows.
__device__ __forceinline__ int sw128_elem(int row, int k, int rows) {
  const int c = k >> 6, kk = k & 63;
  return c * rows * 128 + row * 128 + ((((kk >> 3) ^ (row & 7)) << 4) | ((kk & 7) << 1));
}
// One pass of the float4 merge over features [f0, f0 + 128 NQ): lane l owns f0 + 128 q + 4 l .. + 3. v holds the
// first two segments' rows when the caller issued them; acc = fma(w_s, v_s, acc) over s in order, a = bf16(acc / d).
template <int NQ>
struct VecPass {
  float4 v[2][NQ];
  __device__ __forceinline__ void load(const MergeUpParams& p, const float* base, int n, int s, int f0, int lane) {
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int f = f0 + 128 * q + 4 * lane;
        v[u][q] = (s + u < n && f < p.lv)
                      ? __ldg(reinterpret_cast<const float4*>(base + static_cast<long long>(s + u) * p.ps + f))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
  }
  // v holds segments 0 and 1 on entry
  __device__ __forceinline__ void run(const MergeUpParams& p, const float* base, int n, int f0, int lane, float my_w,
                                      float inv, int j, uint8_t* sB) {
    float4 acc[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < n; s += 2) {
      if (s > 0) load(p, base, n, s, f0, lane);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float w = __shfl_sync(0xffffffffu, my_w, (s + u) & 31);
        if (s + u < n) {
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            acc[q].x = fmaf(w, v[u][q].x, acc[q].x);
            acc[q].y = fmaf(w, v[u][q].y, acc[q].y);
            acc[q].z = fmaf(w, v[u][q].z, acc[q].z);
            acc[q].w = fmaf(w, v[u][q].w, acc[q].w);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int f = f0 + 128 * q + 4 * lane;
      if (f < p.lv) {
        uint2 pk;
        pk.x = pack_bf16(acc[q].x * inv, acc[q].y * inv);
        pk.y = pack_bf16(acc[q].z * inv, acc[q].w * inv);
        *reinterpret_cast<uint2*>(sB + sw128_elem(j, f, kMuReqs)) = pk;   // 4 features: 8 bytes of a 16-byte unit
      }
    }
  }
};

// Merge of request b's n <= 32 segments for head h into row j of the B operand, float4 path (16-byte aligned rows,
// lv % 4 == 0): the same arithmetic and order as the scalar sweep (and belt_merge_segments): m = max of the LSEs,
// d = warp sum of exp(lse_s - m), a = bf16(sum_s exp(lse_s - m) v_s / d) accumulated by fma in segment order. The first
// two segments' rows are loaded together with the LSEs; NQ1 (+ NQ2) float4 columns a lane, two passes for wide rows so
// that two segments stay in flight within the 64 registers a thread has at 1,024 threads.
template <int NQ1, int NQ2>
__device__ __forceinline__ void merge_rows_vec(const MergeUpParams& p, const float* base, int n, int b, int h, int j,
                                               int lane, uint8_t* sB) {
  const float l_me = lane < n ? __ldg(base + static_cast<long long>(lane) * p.ps + p.lv) : -INFINITY;
  VecPass<NQ1> a;
  a.load(p, base, n, 0, 0, lane);
  float m = l_me;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float my_w = lane < n ? __expf(l_me - m) : 0.f;   // lane s: the weight of segment s
  float d = my_w;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  const bool has = d > 0.f;
  const float inv = has ? 1.f / d : 0.f;
  if (lane == 0 && p.lse) p.lse[static_cast<long long>(b) * p.slb + h] = has ? m + __logf(d) : -INFINITY;
  a.run(p, base, n, 0, lane, my_w, inv, j, sB);
  if constexpr (NQ2 > 0) {
    VecPass<NQ2> c;
    c.load(p, base, n, 0, 128 * NQ1, lane);
    c.run(p, base, n, 128 * NQ1, lane, my_w, inv, j, sB);
  }
}
}  // namespace

__global__ void __launch_bounds__(kMuThreads, 1)
    merge_up_kernel(const __grid_constant__ MergeUpMaps maps, const __grid_constant__ MergeUpParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem + kMuOffB;
  float* wts_all = reinterpret_cast<float*>(smem + kMuOffW);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kMuOffBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kMuBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b0 = blockIdx.y * kMuReqs, g = h / p.hpg;
  const int nk = (p.lv + 63) / 64;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kMuBars; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.v);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---------------------------------------------------------------- producer: the first stages, before the merge
  int issued = 0;
  auto produce = [&](int k) {   // thread 0 only; k < kMuStages needs no wait
    const int s = k % kMuStages;
    uint8_t* st = smem + s * kMuStageBytes;
    mbar_arrive_expect_tx(&bars[uFull + s], kMuStageBytes);
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_load_3d(st + q * 8192, &maps.v, &bars[uFull + s], 64 * q, 64 * k, g);
  };
  if (threadIdx.x == 0) {
    for (; issued < nk && issued < kMuStages; ++issued) produce(issued);
    for (int k = issued; k < nk; ++k)
#pragma unroll
      for (int q = 0; q < 4; ++q) tma_prefetch_l2_3d(&maps.v, 64 * q, 64 * k, g);
  }

  // ---------------------------------------------------------------- merge into the B operand
  // zero the operand first: feature columns past r_v must be 0 (U_v's zero-filled rows meet them)
  for (int i = threadIdx.x; i < nk * kMuBChunk / 16; i += kMuThreads)
    reinterpret_cast<uint4*>(sB)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x == 0) allow_dependents_launch();
  // the partials come from the decode kernel ahead of this one, which may still be running (U_v, a weight, was
  // requested above); nothing of this kernel touches global memory other than U_v before this wait
  grid_dependency_wait();
  __syncthreads();
  float* wts = wts_all + warp * kMuWeights;
  {
    const int j = warp, b = b0 + warp;
    if (b < p.num_reqs) {
      const int s0 = __ldg(p.seg_base + b), n = __ldg(p.seg_base + b + 1) - s0;
      const float* base = p.part + static_cast<long long>(s0) * p.ps + static_cast<long long>(h) * p.ph;
      if (p.vec_part && n <= 32) {
        switch ((p.lv + 127) >> 7) {
          case 1: merge_rows_vec<1, 0>(p, base, n, b, h, j, lane, sB); break;
          case 2: merge_rows_vec<2, 0>(p, base, n, b, h, j, lane, sB); break;
          case 3: merge_rows_vec<3, 0>(p, base, n, b, h, j, lane, sB); break;
          case 4: merge_rows_vec<4, 0>(p, base, n, b, h, j, lane, sB); break;
          default: merge_rows_vec<3, 2>(p, base, n, b, h, j, lane, sB); break;
        }
      } else {
      // the segment LSEs' max, then the sum of their exponentials (the order and arithmetic of belt_merge_segments,
      // so that the merged output rounds the same way)
      float m = -INFINITY, my_lse = -INFINITY;
      for (int s = lane; s < n; s += 32) {
        const float l = __ldg(base + static_cast<long long>(s) * p.ps + p.lv);
        if (s == lane) my_lse = l;
        m = fmaxf(m, l);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float d = 0.f;
      for (int s = lane; s < n; s += 32)
        d += __expf((s == lane ? my_lse : __ldg(base + static_cast<long long>(s) * p.ps + p.lv)) - m);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const bool has = d > 0.f;
      const float inv = has ? 1.f / d : 0.f;
      if (lane == 0 && p.lse) p.lse[static_cast<long long>(b) * p.slb + h] = has ? m + __logf(d) : -INFINITY;
      const float my_w = lane < n ? __expf(my_lse - m) : 0.f;   // lane s < 32: the weight of segment s
      for (int f0 = 0; f0 < p.lv; f0 += 32 * 8) {
        float acc[8] = {};
        if (n <= 32) {
          // segment weights from the lanes that loaded them; four segments' rows in flight together
          for (int s4 = 0; s4 < n; s4 += 4) {
            float v[4][8];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float* row = base + static_cast<long long>(s4 + u) * p.ps;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const int f = f0 + 32 * q + lane;
                v[u][q] = (s4 + u < n && f < p.lv) ? __ldg(row + f) : 0.f;
              }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float w = __shfl_sync(0xffffffffu, my_w, (s4 + u) & 31);
#pragma unroll
              for (int q = 0; q < 8; ++q) acc[q] = fmaf(s4 + u < n ? w : 0.f, v[u][q], acc[q]);
            }
          }
        } else {
          for (int sw = 0; sw < n; sw += kMuWeights) {
            const int cnt = min(kMuWeights, n - sw);
            __syncwarp();
            for (int i = lane; i < cnt; i += 32)
              wts[i] = __expf(__ldg(base + static_cast<long long>(sw + i) * p.ps + p.lv) - m);
            __syncwarp();
            for (int i = 0; i < cnt; ++i) {
              const float w = wts[i];
              const float* row = base + static_cast<long long>(sw + i) * p.ps;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const int f = f0 + 32 * q + lane;
                if (f < p.lv) acc[q] = fmaf(w, __ldg(row + f), acc[q]);
              }
            }
          }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int f = f0 + 32 * q + lane;
          if (f < p.lv)
            *reinterpret_cast<__nv_bfloat16*>(sB + sw128_elem(j, f, kMuReqs)) = __float2bfloat16_rn(acc[q] * inv);
        }
      }
      }
    }
  }
  fence_proxy_async_smem();   // the operand's generic-proxy stores, before the tensor core reads them
  __syncthreads();

  // ---------------------------------------------------------------- MMA (thread 32) and the remaining stages (thread 0)
  if (threadIdx.x == 0) {
    bool ok = true;
    for (; ok && issued < nk; ++issued) {
      const int s = issued % kMuStages;
      if (!(ok = mbar_wait(&bars[uEmpty + s], ((issued / kMuStages) - 1) & 1, abort_flag, p.err,
                           kErrTimeoutProducer)))
        break;
      produce(issued);
    }
    if (*abort_flag)
      for (int k = issued > kMuStages ? issued - kMuStages : 0; k < issued; ++k)
        mbar_wait_bounded(&bars[uFull + k % kMuStages], (k / kMuStages) & 1, nullptr, 0, kWaitCycles / 8);
  } else if (threadIdx.x == 32) {
    constexpr uint32_t idesc = idesc_bf16(128, kMuReqs, 1, 0);   // A (U_v^T) MN-major, B (a) K-major
    constexpr uint32_t hiA = desc_hi(1024, kSwizzle128);          // 8 k rows of 128 bytes
    constexpr uint32_t hiB = desc_hi(1024, kSwizzle128);          // 8 request rows
    const uint32_t base = smem_u32(smem), b_base = smem_u32(sB);
    bool ok = true;
    for (int k = 0; k < nk && ok; ++k) {
      const int s = k % kMuStages;
      if (!(ok = mbar_wait(&bars[uFull + s], (k / kMuStages) & 1, abort_flag, p.err, kErrTimeoutMma))) break;
      tc_fence_after();
      const uint32_t st = base + s * kMuStageBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t db = desc_of(desc_lo(b_base + k * kMuBChunk, 16) + 2 * kk, hiB);
#pragma unroll
        for (int half = 0; half < 2; ++half)   // channels [128 half, 128 half + 128): two 64-channel blocks
          mma_ss(tmem + 32 * half, desc_of(desc_lo(st + half * 16384, 8192) + kk * (2048 >> 4), hiA), db, idesc,
                 (k | kk) != 0 ? 1u : 0u);
      }
      mma_commit(&bars[uEmpty + s]);
    }
    if (!ok) *abort_flag = 1;
    mma_commit(&bars[uDone]);   // arrives once every MMA issued has completed
  }
  __syncwarp();

  // ---------------------------------------------------------------- epilogue
  const bool done =
      warp < 4 && __all_sync(0xffffffffu, mbar_wait_bounded(&bars[uDone], 0, p.err, kErrTimeoutEpilogue));
  tc_fence_after();
  __shared__ int staged;
  if (threadIdx.x == 0) staged = 0;
  if (done && !*abort_flag) {
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem);   // [32 requests][256 channels], over stage 0
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_base + 32 * half, r);
      tmem_ld_wait();
      const int ch = 128 * half + 32 * warp + lane;
      if (p.vec_out) {
#pragma unroll
        for (int j = 0; j < kMuReqs; ++j) stg[j * kD + ch] = __float2bfloat16_rn(__uint_as_float(r[j]));
      } else {
#pragma unroll
        for (int j = 0; j < kMuReqs; ++j) {
          const int b = b0 + j;
          if (b < p.num_reqs)
            p.out[static_cast<long long>(b) * p.sot + static_cast<long long>(h) * p.soh + ch] =
                __float2bfloat16_rn(__uint_as_float(r[j]));
        }
      }
    }
    if (threadIdx.x == 0) staged = p.vec_out;
  }
  tc_fence_before();
  __syncthreads();
  if (staged) {   // request j = warp, 8 channels a lane: one 512-byte row a warp
    const int b = b0 + warp;
    if (b < p.num_reqs)
      *reinterpret_cast<uint4*>(p.out + static_cast<long long>(b) * p.sot + static_cast<long long>(h) * p.soh +
                                8 * lane) = reinterpret_cast<const uint4*>(smem)[warp * (kD / 8) + lane];
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

cudaError_t launch_merge_up(const MergeUpMaps& maps, const MergeUpParams& p, cudaStream_t stream) {
  if (p.num_reqs == 0) return cudaSuccess;
  const int smem = 1024 + kMuOffBars + kMuBars * 8 + 16;
  cudaError_t e = cudaFuncSetAttribute(merge_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.nh, (p.num_reqs + kMuReqs - 1) / kMuReqs);
  e = launch_after(merge_up_kernel, grid, dim3(kMuThreads), smem, stream, maps, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace belt
