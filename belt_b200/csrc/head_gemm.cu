// Per-head grouped GEMM on the tensor cores, the operation of the reference's ``_group_gemm``
// (plugins/vllm_lrkv/vllm_lrkv/latent_ops.py:23-44):
//     Out[t, h, n] = sum_k X[t, h, k] * W[g(h), k, n]      (BF16 operands, FP32 accumulation in TMEM, BF16 out)
// for block_diag_query (X = the query [T, 24, 256], W = qmap [4, 256, kq], only the group's column runs computed, the
// other columns written as zeros) and up_project (X = the merged latent output [T, 24, r_v], W = U_v^T [4, r_v, 256]).
//
// One CTA per (128-token tile, head, BN-column tile), 128 threads:
//   * thread 0: TMA producer. Per 64-deep K step one box of X (128 tokens x 64 k, K-major, 128-byte swizzle) and NB
//     boxes of W (64 k x 64 columns, N-contiguous = MN-major, 128-byte swizzle) into a ring of up to 4 stages;
//     rows past T and k past K are zero-filled by the TMA unit;
//   * thread 32: tcgen05 issuer, M = 128 tokens, N = BN, four K = 16 instructions per stage, D in TMEM;
//   * all four warps: epilogue, one token row per thread (TMEM lane), 32 columns per tcgen05.ld, BF16 stores.
// Column tiles that meet no run of the head's group write zeros without touching the tensor cores.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int kHgThreads = 128;
constexpr int kHgABytes = 128 * 128;   // 128 tokens x 64 k x 2 B
constexpr int kHgBBlock = 64 * 128;    // 64 k x 64 columns x 2 B
constexpr int kHgMaxStages = 4;

// The column runs of one group in registers (empty runs as [0, 0)): the epilogue tests columns against them often,
// and the parameter arrays are indexed by the group, which is not a compile-time constant.
struct Runs {
  int lo[3], hi[3];
  __device__ Runs(const HeadGemmParams& p, int g) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const bool v = i < p.nruns[g];
      lo[i] = v ? p.run_lo[g][i] : 0;
      hi[i] = v ? p.run_hi[g][i] : 0;
    }
  }
  __device__ bool live(int n) const {
    return (n >= lo[0] && n < hi[0]) || (n >= lo[1] && n < hi[1]) || (n >= lo[2] && n < hi[2]);
  }
  __device__ bool all_live(int n0, int n1) const {   // [n0, n1) inside one run
    return (lo[0] <= n0 && n1 <= hi[0]) || (lo[1] <= n0 && n1 <= hi[1]) || (lo[2] <= n0 && n1 <= hi[2]);
  }
  __device__ bool all_dead(int n0, int n1) const {   // [n0, n1) meets no run
    return (hi[0] <= n0 || lo[0] >= n1) && (hi[1] <= n0 || lo[1] >= n1) && (hi[2] <= n0 || lo[2] >= n1);
  }
};
}  // namespace

template <int NB>
__global__ void __launch_bounds__(kHgThreads, 1)
    head_gemm_kernel(const __grid_constant__ HeadGemmMaps maps, const __grid_constant__ HeadGemmParams p) {
  constexpr int BN = 64 * NB;
  constexpr int kStageBytes = kHgABytes + NB * kHgBBlock;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.stages * kStageBytes);   // full[S], empty[S], done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kHgMaxStages + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * 128, h = blockIdx.y, g = h / p.hpg, n0 = blockIdx.z * BN;
  const int row = t0 + threadIdx.x;   // this thread's token in the epilogue
  __nv_bfloat16* out_row = p.Out + static_cast<long long>(row) * p.sot + static_cast<long long>(h) * p.soh;

  const Runs runs(p, g);
  // X comes from the kernel ahead of this one, which may still be running, and Out may reuse memory it reads: wait for
  // it before any global access but the weights'
  if (threadIdx.x == 0) allow_dependents_launch();
  if (runs.all_dead(n0, n0 + BN)) {   // no live column: zeros (uniform over the CTA, before any barrier or TMEM use)
    grid_dependency_wait();
    if (row < p.T) {
      if (p.vec_out && n0 + BN <= p.N) {
        uint4* dst = reinterpret_cast<uint4*>(out_row + n0);
#pragma unroll
        for (int q = 0; q < BN / 8; ++q) dst[q] = make_uint4(0u, 0u, 0u, 0u);
      } else {
        for (int c = 0; c < BN && n0 + c < p.N; ++c) out_row[n0 + c] = __float2bfloat16_rn(0.f);
      }
    }
    return;
  }

  const int nk = (p.K + 63) / 64;
  const int S = p.stages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars[s], 1);
      mbar_init(&bars[kHgMaxStages + s], 1);
    }
    mbar_init(&bars[2 * kHgMaxStages], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.x);
    tma_prefetch_desc(&maps.w);
  }
  if (warp == 1) tmem_alloc(tmem_slot, BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    // ---------------------------------------------------------------- producer
    grid_dependency_wait();
    int issued = 0;
    for (int k = 0; k < nk; ++k) {
      const int s = k % S;
      if (k >= S && !mbar_wait(&bars[kHgMaxStages + s], ((k / S) - 1) & 1, abort_flag, p.err, kErrTimeoutProducer)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* st = smem + s * kStageBytes;
      mbar_arrive_expect_tx(&bars[s], kStageBytes);
      tma_load_3d(st, &maps.x, &bars[s], k * 64, h, t0);
#pragma unroll
      for (int b = 0; b < NB; ++b) tma_load_3d(st + kHgABytes + b * kHgBBlock, &maps.w, &bars[s], n0 + 64 * b, k * 64, g);
      ++issued;
    }
    if (*abort_flag)   // let the copies already issued land before the CTA's shared memory goes away
      for (int k = issued > S ? issued - S : 0; k < issued; ++k)
        mbar_wait_bounded(&bars[k % S], (k / S) & 1, nullptr, 0, kWaitCycles / 8);
  } else if (threadIdx.x == 32) {
    // ---------------------------------------------------------------- tcgen05 issuer
    constexpr uint32_t idesc = idesc_bf16(128, BN, 0, 1);      // A K-major, B MN-major
    constexpr uint32_t hiA = desc_hi(1024, kSwizzle128);        // 8 token rows = 1 KB
    constexpr uint32_t hiB = desc_hi(1024, kSwizzle128);        // 8 k rows = 1 KB
    const uint32_t base = smem_u32(smem);
    bool ok = true;
    for (int k = 0; k < nk && ok; ++k) {
      const int s = k % S;
      if (!(ok = mbar_wait(&bars[s], (k / S) & 1, abort_flag, p.err, kErrTimeoutMma))) break;
      tc_fence_after();
      const uint32_t a = base + s * kStageBytes;
      uint64_t da = desc_of(desc_lo(a, 16), hiA);
      uint64_t db = desc_of(desc_lo(a + kHgABytes, kHgBBlock), hiB);   // LBO: the next 64-column block
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        mma_ss(tmem, da, db, idesc, (k | kk) != 0 ? 1u : 0u);
        da += 2;           // 16 k = 32 bytes along the swizzled row
        db += 2048 >> 4;   // 16 k rows = 2 KB
      }
      mma_commit(&bars[kHgMaxStages + s]);
    }
    if (ok) {
      mma_commit(&bars[2 * kHgMaxStages]);
    } else {
      *abort_flag = 1;
      mma_commit(&bars[2 * kHgMaxStages]);   // arrives once the MMAs already issued are done
    }
  }
  __syncwarp();

  // -------------------------------------------------------------------- epilogue
  const bool done = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[2 * kHgMaxStages], 0, p.err, kErrTimeoutEpilogue));
  tc_fence_after();
  if (done && !*abort_flag) {
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c0, r);
      tmem_ld_wait();
      if (row >= p.T) continue;
      const int nb = n0 + c0;
      // per 8 columns: one 16-byte store when they are all live (values) or all dead (zeros) and inside the row
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int n8 = nb + 8 * q;
        const bool live8 = runs.all_live(n8, n8 + 8), dead8 = runs.all_dead(n8, n8 + 8);
        if ((live8 || dead8) && n8 + 8 <= p.N && p.vec_out) {
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (live8) {
            v.x = pack_bf16(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
            v.y = pack_bf16(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
            v.z = pack_bf16(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
            v.w = pack_bf16(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
          }
          *reinterpret_cast<uint4*>(out_row + n8) = v;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int n = n8 + i;
            if (n < p.N) out_row[n] = __float2bfloat16_rn(runs.live(n) ? __uint_as_float(r[8 * q + i]) : 0.f);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

int head_gemm_smem_bytes(int nb, int stages) {
  return 1024 + stages * (kHgABytes + nb * kHgBBlock) + (2 * kHgMaxStages + 1) * 8 + 16;
}

cudaError_t launch_head_gemm(const HeadGemmMaps& maps, HeadGemmParams p, cudaStream_t stream) {
  if (p.T == 0) return cudaSuccess;
  const int nk = (p.K + 63) / 64;
  p.stages = nk < kHgMaxStages ? nk : kHgMaxStages;
  const int smem = head_gemm_smem_bytes(p.nb, p.stages);
  dim3 grid((p.T + 127) / 128, p.G * p.hpg, (p.N + 64 * p.nb - 1) / (64 * p.nb));
  cudaError_t e;
  switch (p.nb) {
    case 1:
      e = cudaFuncSetAttribute(head_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      e = launch_after(head_gemm_kernel<1>, grid, dim3(kHgThreads), smem, stream, maps, p);
      break;
    case 2:
      e = cudaFuncSetAttribute(head_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      e = launch_after(head_gemm_kernel<2>, grid, dim3(kHgThreads), smem, stream, maps, p);
      break;
    case 4:
      e = cudaFuncSetAttribute(head_gemm_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      e = launch_after(head_gemm_kernel<4>, grid, dim3(kHgThreads), smem, stream, maps, p);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace belt
