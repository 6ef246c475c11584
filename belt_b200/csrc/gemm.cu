// Dense BF16 GEMM on the tensor cores: C[M, N] = A[M, K] * B[N, K]^T (both operands K-major, FP32 accumulation in
// TMEM, BF16 out), the model-side linear layers around the latent attention (plugins/vllm_lrkv/vllm_lrkv/models/
// qwen3_5_latent.py:130-140, 204-217: q_gate_proj, o_proj, and kv_latent_proj at prefill sizes).
//
// Persistent grid (one CTA per SM, tiles BM = 128 x BN = 128 or 256, taken round-robin), 192 threads:
//   * warp 0 (one thread): TMA producer, per 64-deep K block one box of A (128 rows x 64) and one of B (BN rows x 64),
//     both K-major with the 128-byte swizzle, into a ring of 4-6 stages (zeros past M, N and K);
//   * warp 1 (one thread): tcgen05 issuer, M = 128, N = BN, K = 16 per instruction, into one of two TMEM accumulators
//     (2 x BN columns), so that tile i's epilogue overlaps tile i + 1's MMAs;
//   * warps 2-5: epilogue, one row per thread (warp w reads TMEM lanes 32 (w % 4) ..), 32 columns per tcgen05.ld,
//     BF16 rounding and 16-byte stores.
// Every wait is bounded (common.cuh): a timed-out wait records a code in the error word, the roles drain what they
// issued and the CTA exits.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int kGmThreads = 192;
constexpr int kGmABytes = 128 * 128;   // 128 rows x 64 k x 2 B
constexpr int kGmMaxStages = 6;
constexpr int kGmRing = 196608;        // 192 KB of stages
// barriers: full[6], empty[6], acc_full[2], acc_empty[2], drain
constexpr int gFull = 0, gEmpty = 6, gAccFull = 12, gAccEmpty = 14, gDrain = 16, kGmBars = 17;
}  // namespace

template <int BN>
__global__ void __launch_bounds__(kGmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ GemmMaps maps, const __grid_constant__ GemmParams p) {
  constexpr int kBBytes = BN * 128;
  constexpr int kStage = kGmABytes + kBBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGmRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kGmBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  const int nk = (p.K + 63) / 64;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGmMaxStages; ++i) {
      mbar_init(&bars[gFull + i], 1);
      mbar_init(&bars[gEmpty + i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[gAccFull + i], 1);
      mbar_init(&bars[gAccEmpty + i], 4);
    }
    mbar_init(&bars[gDrain], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.a);
    tma_prefetch_desc(&maps.b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int fill = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        const int m0 = (t % p.tiles_m) * 128, n0 = (t / p.tiles_m) * BN;
        for (int k = 0; k < nk; ++k, ++fill) {
          const int s = fill % S;
          if (fill >= S && !(ok = mbar_wait(&bars[gEmpty + s], ((fill / S) - 1) & 1, abort_flag, p.err,
                                            kErrTimeoutProducer)))
            break;
          uint8_t* st = smem + s * kStage;
          mbar_arrive_expect_tx(&bars[gFull + s], kStage);
          tma_load_2d(st, &maps.a, &bars[gFull + s], k * 64, m0);
          tma_load_2d(st + kGmABytes, &maps.b, &bars[gFull + s], k * 64, n0);
        }
      }
      if (*abort_flag)   // let the copies already issued land before the shared memory goes away
        for (int f = fill > S ? fill - S : 0; f < fill; ++f)
          mbar_wait_bounded(&bars[gFull + f % S], (f / S) & 1, nullptr, 0, kWaitCycles / 8);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ tcgen05 issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, BN, 0, 0);   // both operands K-major
      constexpr uint32_t hi = desc_hi(1024, kSwizzle128);     // 8 rows of 128 bytes = 1 KB
      const uint32_t base = smem_u32(smem);
      int fill = 0, j = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !(ok = mbar_wait(&bars[gAccEmpty + b], ((j >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutMma)))
          break;
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        for (int k = 0; k < nk; ++k, ++fill) {
          const int s = fill % S;
          if (!(ok = mbar_wait(&bars[gFull + s], (fill / S) & 1, abort_flag, p.err, kErrTimeoutMma))) break;
          tc_fence_after();
          const uint32_t a = base + s * kStage;
          const uint32_t la = desc_lo(a, 16), lb = desc_lo(a + kGmABytes, 16);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ss(d, desc_of(la + 2 * kk, hi), desc_of(lb + 2 * kk, hi), idesc, (k | kk) != 0 ? 1u : 0u);
          mma_commit(&bars[gEmpty + s]);
        }
        if (ok) mma_commit(&bars[gAccFull + b]);
      }
      if (*abort_flag) {   // wait for the MMAs already issued before TMEM goes away
        mma_commit(&bars[gDrain]);
        mbar_wait_bounded(&bars[gDrain], 0, nullptr, 0, kWaitCycles / 8);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int quad = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    int j = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++j) {
      const int b = j & 1;
      const bool got = mbar_wait(&bars[gAccFull + b], (j >> 1) & 1, abort_flag, p.err, kErrTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int m0 = (t % p.tiles_m) * 128, n0 = (t / p.tiles_m) * BN;
      const int row = m0 + quad * 32 + lane;
      __nv_bfloat16* out = p.c + static_cast<long long>(row) * p.ldc + n0;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + b * BN + c0, r);
        tmem_ld_wait();
        if (row >= p.M || n0 + c0 >= p.N) continue;
        if (p.vec_out && n0 + c0 + 32 <= p.N) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
            v.y = pack_bf16(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
            v.z = pack_bf16(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
            v.w = pack_bf16(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
            *reinterpret_cast<uint4*>(out + c0 + 8 * q) = v;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (n0 + c0 + i < p.N) out[c0 + i] = __float2bfloat16_rn(__uint_as_float(r[i]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[gAccEmpty + b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

cudaError_t launch_gemm(const GemmMaps& maps, GemmParams p, int num_sms, cudaStream_t stream) {
  if (p.M == 0 || p.N == 0) return cudaSuccess;
  const int smem = 1024 + kGmRing + kGmBars * 8 + 16;
  cudaError_t e;
  if (p.bn == 256) {
    p.stages = kGmRing / (kGmABytes + 256 * 128);   // 4
    e = cudaFuncSetAttribute(gemm_bf16_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    gemm_bf16_kernel<256><<<p.num_tiles < num_sms ? p.num_tiles : num_sms, kGmThreads, smem, stream>>>(maps, p);
  } else {
    p.stages = kGmRing / (kGmABytes + 128 * 128);   // 6
    e = cudaFuncSetAttribute(gemm_bf16_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    gemm_bf16_kernel<128><<<p.num_tiles < num_sms ? p.num_tiles : num_sms, kGmThreads, smem, stream>>>(maps, p);
  }
  return cudaGetLastError();
}

}  // namespace belt
