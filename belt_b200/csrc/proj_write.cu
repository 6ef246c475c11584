// Fused latent cache write: down-projection of the new tokens' inputs into the cache row, the RMS fold of every K
// group and the paged scatter, in one kernel. It replaces the model-side ``kv_latent_proj`` linear
// (plugins/vllm_lrkv/vllm_lrkv/models/qwen3_5_latent.py:139-140, 213; weight layout lrkv/runtime/export_latent.py:
// 193-205) followed by ``latent_rows_to_cache`` (plugins/vllm_lrkv/vllm_lrkv/latent_ops.py:85-158):
//     c      = bf16(x @ W_down^T)                      x [T, hidden], W_down [W, hidden] (zero rows at the gaps)
//     k_pre  = U_g c_g  (FP32)                         per KV group, its latent columns (one or two runs)
//     row    = [bf16(c_g * rsqrt(mean(k_pre^2) + eps)) per group | c[lk:W]]   at cache[slot]; slot < 0 skipped
//
// One CTA (128 threads) per 128-token tile and work item: KV group g (items 0..G-1) or up to four 64-column chunks of
// the V part [lk, W). An item's cache columns are covered by at most five 64-column chunks (its "window").
//   phase 1: thread 0 streams, per 64-deep hidden step, the x tile (128 tokens x 64, K-major) and the window's
//            W_down rows (64 x 64 per chunk, K-major) through a 3-stage ring; thread 32 issues tcgen05 MMAs
//            D1[token, window column] (N = 64 per chunk, <= 256 per instruction) into TMEM;
//   epilogue 1 (all threads, one token per thread): c = bf16(D1); a V item writes c to the cache row; a group item
//            zeroes the window columns outside its runs and stores c as the K-major A tile of phase 2;
//   phase 2 (groups): k_pre[token, channel] = c_window . u_cat[window rows, g*256 + channel] (N = 256, u_cat read
//            MN-major; rows of other groups meet zeros in A, rows past lk are zero-filled by TMA);
//   epilogue 2: rho from the 256 channels, the group's runs scaled and written to the cache row.
// In c-input mode (``latent_rows_to_cache``, latent_ops.py:138-158: the model computed c) phase 1 is skipped and
// epilogue 1 reads the window columns of c from global memory; phase 2 and epilogue 2 are the same, so the RMS fold
// runs on the tensor cores at every batch size.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int kPwThreads = 128;
constexpr int kPwXBytes = 128 * 128;                  // 128 tokens x 64 hidden
constexpr int kPwChunkBytes = 64 * 128;               // 64 rows x 64 hidden
// Phase-1 ring of 3 stages of the widest window (x tile + 5 chunks). Stages sized to the item's window (4-7 stages in
// 224 KB) were measured no faster: phase 1 is bound by the SM's inflow of 128-byte rows (~70 GB/s), not by latency.
constexpr int kPwStage = kPwXBytes + kPwMaxChunks * kPwChunkBytes;   // 56 KB
constexpr int kPwStages = 3;
constexpr int kPwRing = kPwStages * kPwStage;
constexpr int kPwA2 = 0;                              // phase-2 A tile, 16 KB per chunk, over the ring
constexpr int kPwB2 = kPwMaxChunks * kPwXBytes;       // phase-2 B stages: 2 x (64 rows x 256 channels)
constexpr int kPwB2Stage = 4 * kPwChunkBytes;         // 32 KB
static_assert(kPwB2 + 2 * kPwB2Stage <= kPwRing, "phase-2 tiles exceed the ring");
// barriers
constexpr int pFull = 0, pEmpty = 3, pDone1 = 6, pA2 = 7, pFull2 = 8, pEmpty2 = 10, pDone2 = 12, kPwBars = 13;

__device__ __forceinline__ long long pw_slot(const ProjWriteParams& p, int t) {
  long long s = p.slots_i64 ? static_cast<const long long*>(p.slots)[t]
                            : static_cast<long long>(static_cast<const int32_t*>(p.slots)[t]);
  return (s >= 0 && s < p.num_slots) ? s : -1;
}



// Offset of 16-byte unit `u` (8 columns) of token row `r` in a K-major 128-byte-swizzled tile.
__device__ __forceinline__ int sw128(int r, int u) { return r * 128 + ((u ^ (r & 7)) << 4); }
}  // namespace

__global__ void __launch_bounds__(kPwThreads, 1)
    proj_write_kernel(const __grid_constant__ ProjWriteMaps maps, const __grid_constant__ ProjWriteParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPwRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kPwBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * 128, item = blockIdx.y;
  const bool group = item < p.G;
  const int g = item;
  // the group's two runs in registers (the epilogues test many columns; the arrays are indexed by the item)
  const int a_lo = group ? p.a_lo[g] : 0, a_hi = group ? a_lo + p.a_n[g] : 0;
  const int b_lo = group ? p.b_lo[g] : 0, b_hi = group ? b_lo + p.b_n[g] : 0;
  // Bit j set: column cb + j of a 32-column window lies in one of the group's runs. The window is the same for every
  // thread, so the mask is computed once per window and applied to the packed words without a branch per column (a
  // test per column cost ~1,500 cycles per window, most of epilogue 1).
  auto run_mask = [&](int cb) -> uint32_t {
    auto span = [&](int lo, int hi) -> uint32_t {
      const int l = max(lo - cb, 0), h = min(hi - cb, 32);
      if (h <= l) return 0u;
      return (h - l == 32 ? 0xFFFFFFFFu : (1u << (h - l)) - 1u) << l;
    };
    return span(a_lo, a_hi) | span(b_lo, b_hi);
  };
  // the packed word j (columns cb + 2j, cb + 2j + 1) with the halves outside the runs zeroed
  auto keep_word = [](uint32_t m, int j) -> uint32_t {
    return ((0u - ((m >> (2 * j)) & 1u)) & 0x0000FFFFu) | ((0u - ((m >> (2 * j + 1)) & 1u)) & 0xFFFF0000u);
  };
  const int nch = p.item_nch[item];
  const int win_lo = p.item_chunk[item][0];
  const bool win_contig = p.item_chunk[item][nch - 1] - win_lo == nch - 1;
  const int row = t0 + threadIdx.x;
  const long long slot = row < p.T ? pw_slot(p, row) : -1;
  __nv_bfloat16* dst = slot >= 0 ? p.cache + (slot / p.page) * p.sblk + (slot % p.page) * p.stok : nullptr;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPwBars; ++i) mbar_init(&bars[i], i == pA2 ? kPwThreads : 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (!p.c_in) {
      tma_prefetch_desc(&maps.x);
      tma_prefetch_desc(&maps.w);
    }
    tma_prefetch_desc(&maps.u);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const int nk = (p.hidden + 63) / 64;
  const uint32_t base = smem_u32(smem);

  // ------------------------------------------------------------------ phase 1 (roles)
  if (p.c_in) {
    // c is given: nothing to compute
  } else if (threadIdx.x == 0) {
    int issued = 0;
    for (int k = 0; k < nk; ++k) {
      const int s = k % kPwStages;
      if (k >= kPwStages && !mbar_wait(&bars[pEmpty + s], ((k / kPwStages) - 1) & 1, abort_flag, p.err,
                                       kErrTimeoutProducer)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* st = smem + s * kPwStage;
      mbar_arrive_expect_tx(&bars[pFull + s], kPwXBytes + nch * kPwChunkBytes);
      tma_load_2d(st, &maps.x, &bars[pFull + s], k * 64, t0);
      for (int i = 0; i < nch; ++i)
        tma_load_2d(st + kPwXBytes + i * kPwChunkBytes, &maps.w, &bars[pFull + s], k * 64, 64 * p.item_chunk[item][i]);
      ++issued;
    }
    if (*abort_flag)
      for (int k = issued > kPwStages ? issued - kPwStages : 0; k < issued; ++k)
        mbar_wait_bounded(&bars[pFull + k % kPwStages], (k / kPwStages) & 1, nullptr, 0, kWaitCycles / 8);
  } else if (threadIdx.x == 32) {
    constexpr uint32_t hiSw = desc_hi(1024, kSwizzle128);
    const int n1 = nch > 4 ? 256 : 64 * nch;
    const uint32_t id1 = idesc_bf16(128, n1, 0, 0);
    constexpr uint32_t id1b = idesc_bf16(128, 64, 0, 0);
    bool ok = true;
    for (int k = 0; k < nk && ok; ++k) {
      const int s = k % kPwStages;
      if (!(ok = mbar_wait(&bars[pFull + s], (k / kPwStages) & 1, abort_flag, p.err, kErrTimeoutMma))) break;
      tc_fence_after();
      const uint32_t st = base + s * kPwStage;
      uint64_t da = desc_of(desc_lo(st, 16), hiSw);
      uint64_t db = desc_of(desc_lo(st + kPwXBytes, 16), hiSw);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t acc = (k | kk) != 0 ? 1u : 0u;
        mma_ss(tmem, da, db, id1, acc);
        if (nch > 4) mma_ss(tmem + 256, da, db + ((4 * kPwChunkBytes) >> 4), id1b, acc);
        da += 2;
        db += 2;
      }
      mma_commit(&bars[pEmpty + s]);
    }
    if (!ok) *abort_flag = 1;
    mma_commit(&bars[pDone1]);
  }
  __syncwarp();

  const bool done1 =
      p.c_in || __all_sync(0xffffffffu, mbar_wait_bounded(&bars[pDone1], 0, p.err, kErrTimeoutEpilogue));
  tc_fence_after();
  const bool live = done1 && !*abort_flag;
  // phase-2 operands for the first two chunks can stream in while epilogue 1 runs (the ring is free now)
  if (group && live && threadIdx.x == 0) {
    for (int i = 0; i < nch && i < 2; ++i) {
      mbar_arrive_expect_tx(&bars[pFull2 + i], kPwB2Stage);
#pragma unroll
      for (int nb = 0; nb < 4; ++nb)
        tma_load_2d(smem + kPwB2 + i * kPwB2Stage + nb * kPwChunkBytes, &maps.u, &bars[pFull2 + i],
                    g * kD + 64 * nb, 64 * p.item_chunk[item][i]);
    }
  }

  __syncwarp();
  // ------------------------------------------------------------------ epilogue 1: c = bf16(D1), or c itself
  const __nv_bfloat16* crow = p.c_in && row < p.T ? p.c + static_cast<long long>(row) * p.sct : nullptr;
  if (live) {
    for (int i = 0; i < nch; ++i) {
      const int col0 = 64 * p.item_chunk[item][i];
      uint32_t v[32];
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[16];
        const int cb = col0 + 32 * half;
        if (p.c_in) {
          // 32 columns of this token's c row (zeros past W or past the last token)
          if (crow && p.c_vec && cb + 32 <= p.W) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint4 w = __ldg(reinterpret_cast<const uint4*>(crow + cb + 8 * u));
              pk[4 * u] = w.x;
              pk[4 * u + 1] = w.y;
              pk[4 * u + 2] = w.z;
              pk[4 * u + 3] = w.w;
            }
          } else {
            const uint16_t* cr = reinterpret_cast<const uint16_t*>(crow);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t lo = crow && cb + 2 * j < p.W ? cr[cb + 2 * j] : 0u;
              const uint32_t hi = crow && cb + 2 * j + 1 < p.W ? cr[cb + 2 * j + 1] : 0u;
              pk[j] = lo | (hi << 16);
            }
          }
          if (group) {
            const uint32_t m = run_mask(cb);
#pragma unroll
            for (int j = 0; j < 16; ++j) pk[j] &= keep_word(m, j);
          }
        } else {
          tmem_ld32(tmem + lane_base + 64 * i + 32 * half, v);
          tmem_ld_wait();
          const uint32_t m = group ? run_mask(cb) : 0xFFFFFFFFu;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            pk[j] = pack_bf16(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1])) & keep_word(m, j);
        }
        if (group) {
          uint8_t* a2 = smem + kPwA2 + i * kPwXBytes;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(a2 + sw128(threadIdx.x, 4 * half + u)) =
                make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        } else if (dst) {
          for (int u = 0; u < 4; ++u) {
            const int c = col0 + 32 * half + 8 * u;
            if (c >= p.lk && c + 8 <= p.W && p.vec_ok) {
              *reinterpret_cast<uint4*>(dst + c) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
            } else {
              for (int e = 0; e < 8; ++e) {
                if (c + e < p.lk || c + e >= p.W) continue;
                const uint32_t w2 = pk[4 * u + (e >> 1)];
                const uint16_t bits = (e & 1) ? static_cast<uint16_t>(w2 >> 16) : static_cast<uint16_t>(w2 & 0xFFFFu);
                reinterpret_cast<uint16_t*>(dst)[c + e] = bits;
              }
            }
          }
        }
      }
    }
  }

  if (group) {
    fence_proxy_async_smem();   // A tile written by the generic proxy, read by the tensor cores
    tc_fence_before();
    mbar_arrive(&bars[pA2]);
    // ---------------------------------------------------------------- phase 2 (roles)
    if (threadIdx.x == 0 && live) {
      for (int i = 2; i < nch; ++i) {
        const int s = i & 1;
        if (!mbar_wait(&bars[pEmpty2 + s], ((i >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutProducer)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&bars[pFull2 + s], kPwB2Stage);
#pragma unroll
        for (int nb = 0; nb < 4; ++nb)
          tma_load_2d(smem + kPwB2 + s * kPwB2Stage + nb * kPwChunkBytes, &maps.u, &bars[pFull2 + s],
                      g * kD + 64 * nb, 64 * p.item_chunk[item][i]);
      }
    } else if (threadIdx.x == 32) {
      bool ok = live && mbar_wait(&bars[pA2], 0, abort_flag, p.err, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        constexpr uint32_t hiSw = desc_hi(1024, kSwizzle128);
        constexpr uint32_t id2 = idesc_bf16(128, 256, 0, 1);   // A K-major, B (u_cat) MN-major
        for (int i = 0; i < nch && ok; ++i) {
          const int s = i & 1;
          if (!(ok = mbar_wait(&bars[pFull2 + s], (i >> 1) & 1, abort_flag, p.err, kErrTimeoutMma))) break;
          tc_fence_after();
          uint64_t da = desc_of(desc_lo(base + kPwA2 + i * kPwXBytes, 16), hiSw);
          uint64_t db = desc_of(desc_lo(base + kPwB2 + s * kPwB2Stage, kPwChunkBytes), hiSw);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_ss(tmem, da, db, id2, (i | kk) != 0 ? 1u : 0u);
            da += 2;
            db += 2048 >> 4;
          }
          mma_commit(&bars[pEmpty2 + s]);
        }
      }
      if (!ok) *abort_flag = 1;
      mma_commit(&bars[pDone2]);
    }
    __syncwarp();
    const bool done2 = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[pDone2], 0, p.err, kErrTimeoutEpilogue));
    tc_fence_after();
    // ---------------------------------------------------------------- epilogue 2: rho, scaled runs
    if (done2 && !*abort_flag) {
      // sum of squares over the 256 channels in four interleaved partial sums (one dependent chain of 256 FMAs was
      // ~1,000 cycles of latency)
      float ss4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t v[32];
      for (int c0 = 0; c0 < kD; c0 += 32) {
        tmem_ld32(tmem + lane_base + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) ss4[j & 3] = fmaf(__uint_as_float(v[j]), __uint_as_float(v[j]), ss4[j & 3]);
      }
      const float ss = (ss4[0] + ss4[1]) + (ss4[2] + ss4[3]);
      const float inv = rsqrtf(ss / kD + p.eps);
      if (dst) {
        const uint8_t* a2 = smem + kPwA2;
        for (int run = 0; run < 2; ++run) {
          const int lo = run ? b_lo : a_lo, n = run ? b_hi - b_lo : a_hi - a_lo;
          int c = lo;
          while (c < lo + n) {
            // window position of column c (the window's chunks ascend; contiguous windows need no search)
            int i = (c >> 6) - win_lo;
            if (!win_contig) {
              i = 0;
              while (i + 1 < nch && p.item_chunk[item][i] != (c >> 6)) ++i;
            }
            const int j = c & 63;
            const uint8_t* unit = a2 + i * kPwXBytes + sw128(threadIdx.x, j >> 3);
            if ((c & 7) == 0 && c + 8 <= lo + n && p.vec_ok) {
              const uint4 w = *reinterpret_cast<const uint4*>(unit);
              const uint32_t in[4] = {w.x, w.y, w.z, w.w};
              uint32_t o[4];
#pragma unroll
              for (int q = 0; q < 4; ++q)
                o[q] = pack_bf16(__uint_as_float(in[q] << 16) * inv, __uint_as_float(in[q] & 0xFFFF0000u) * inv);
              *reinterpret_cast<uint4*>(dst + c) = make_uint4(o[0], o[1], o[2], o[3]);
              c += 8;
            } else {
              const uint16_t bits = reinterpret_cast<const uint16_t*>(unit)[j & 7];
              const float x = __uint_as_float(static_cast<uint32_t>(bits) << 16) * inv;
              dst[c] = __float2bfloat16_rn(x);
              c += 1;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int proj_write_smem_bytes() { return 1024 + kPwRing + kPwBars * 8 + 16; }

cudaError_t launch_proj_write(const ProjWriteMaps& maps, const ProjWriteParams& p, cudaStream_t stream) {
  if (p.T == 0) return cudaSuccess;
  const int smem = proj_write_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(proj_write_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + 127) / 128, p.n_items);
  proj_write_kernel<<<grid, kPwThreads, smem, stream>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace belt
