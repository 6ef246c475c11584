// Single-pass paged latent decode for sm_100a (tcgen05 + TMEM + TMA), split-KV over a persistent grid.
//
// Replaces the reference's Hopper CuTe kernel ``LatentDecodeSm90`` (plugins/vllm_lrkv/vllm_lrkv/cute_decode.py:90-484)
// with a Blackwell design:
//
// * one CTA per SM walks the segments the schedule dealt it (cute_decode.py:571-598 semantics, 128-token tiles);
// * warp 0 streams the cache through a ring of 32 KB stages = [128 tokens x 128 features] as two SWIZZLE_128B
//   halves of [128 x 64]; a tile is the K part's pairs (columns [0, n_k * 64)) then the V part's pairs (columns
//   v_offset + [0, r_v)); pages of 16..128 tokens are fetched as boxes of `page` rows through a 3-D tensor map
//   over the (possibly strided) [blocks, page, W] cache view; pages past the request read as zeros (OOB boxes);
// * warp 1 (one thread) issues tcgen05.mma, M = 128 tokens:
//     - scores S[tok, head] (N = 32: 24 heads + 8 zero rows) over the K part against the block-diagonal query;
//     - the rebuilt RoPE keys gain * B_g c~_g: per group the 16-column K-steps holding its rr_g coordinates
//       against resident [64 x 16] images of the rope blocks (N = 64) into TMEM;
//     - after the epilogue rotated the keys (BF16, back into TMEM), the RoPE score with A read from TMEM;
//     - O^T[latent, head] += V^T P per 128-latent block (A = the cache stage read MN-major, B = P from shared memory);
// * warps 2-5 (128 threads = the 128 TMEM lanes): RoPE rotation of the rebuilt keys (BF16 round, fp32 rotation,
//   BF16 operand: cute_decode.py:473-484), masked online softmax in the exp2 domain with lazy rescaling of O
//   (only when a head's running max grows by more than 2^8; the final normalisation makes it exact), P rounded to
//   BF16 (cute_decode.py:408), and the per-segment epilogue: normalised partial output and natural-log LSE
//   (cute_decode.py:435-455).
//
// TMEM columns: [0, 64) two S buffers, [64, 320) the four groups' rebuilt keys (fp32; the rotated BF16 keys are
// packed into the first 32 columns of each group's range), [320, 320 + 32 * n_vp) the O^T blocks.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace dec {
constexpr int kTile = 128;
constexpr int kStages = 3;
constexpr int kHalfBytes = kTile * 64 * 2;      // [128 x 64] BF16 = 16 KB
constexpr int kStageBytes = 2 * kHalfBytes;     // 32 KB
constexpr int kQChunkBytes = 32 * 64 * 2;       // [32 x 64] BF16 = 4 KB
constexpr int kMaxQChunks = 16;                 // n_k + 4 <= 16
constexpr int kKstBytes = 64 * 16 * 2;          // [64 x 16] BF16 = 2 KB
constexpr int kPBytes = kTile * 32 * 2;         // [128 tokens x 32 heads] BF16 = 8 KB
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kTmemK = 64;
constexpr int kTmemO = 320;

constexpr int kOffRing = 0;
constexpr int kOffQ = kOffRing + kStages * kStageBytes;
constexpr int kOffB = kOffQ + kMaxQChunks * kQChunkBytes;
constexpr int kOffP = kOffB + kDecodeMaxKsteps * kKstBytes;
constexpr int kOffRedMax = kOffP + 2 * kPBytes;        // [2][4][32] fp32
constexpr int kOffRedSum = kOffRedMax + 2 * 4 * 32 * 4; // [4][32] fp32
constexpr int kOffBars = kOffRedSum + 4 * 32 * 4;
constexpr int kNumBars = 32;
constexpr int kOffMisc = kOffBars + kNumBars * 8;
constexpr int kSmemUsed = kOffMisc + 16;
constexpr int kSmemBytes = kSmemUsed + 1024;           // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");

// barrier indices
constexpr int bFull = 0;                   // [kStages]
constexpr int bEmpty = bFull + kStages;    // [kStages]
constexpr int bQFull = bEmpty + kStages;
constexpr int bQEmpty = bQFull + 1;
constexpr int bKrawFull = bQEmpty + 1;
constexpr int bKpeFull = bKrawFull + 1;
constexpr int bSFull = bKpeFull + 1;       // [2]
constexpr int bSFree = bSFull + 2;         // [2]
constexpr int bPFull = bSFree + 2;         // [2]
constexpr int bPvDone = bPFull + 2;        // [2]
constexpr int bOFree = bPvDone + 2;
constexpr int bDrain = bOFree + 1;
constexpr int bEpi = bDrain + 1;           // epilogue group barrier (4 warps), replaces bar.sync so waits stay bounded
static_assert(bEpi < kNumBars, "barriers");
}  // namespace dec

struct SegmentInfo {
  int b, t0, t1, end;
  bool ok;
};

__device__ __forceinline__ SegmentInfo load_segment(const DecodeParams& p, int s) {
  SegmentInfo si;
  si.b = __ldg(p.work + 4 * s);
  si.t0 = __ldg(p.work + 4 * s + 1);
  si.t1 = __ldg(p.work + 4 * s + 2);
  si.ok = si.b >= 0 && si.b < p.num_reqs && si.t0 >= 0 && si.t1 > si.t0;
  int seq = si.ok ? __ldg(p.seq_lens + si.b) : 0;
  si.ok = si.ok && (si.t1 - 1) * dec::kTile < seq;
  si.end = min(si.t1 * dec::kTile, seq);
  return si;
}

__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles / 8) return false;
  }
  return true;
}

// Element i (BF16) of 8 x 16 bytes held in registers, as fp32 (i is a compile-time constant after unrolling).
__device__ __forceinline__ float bf16_lane(const uint4 (&v)[8], int i) {
  const uint4 q = v[i >> 3];
  const int wi = (i >> 1) & 3;
  const uint32_t w = wi == 0 ? q.x : wi == 1 ? q.y : wi == 2 ? q.z : q.w;
  return __uint_as_float((i & 1) ? (w & 0xFFFF0000u) : (w << 16));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(dec::kThreads, 1)
    latent_decode_kernel(const __grid_constant__ CUtensorMap tm_cache, const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ DecodeParams p) {
  using namespace dec;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem + kOffRing;
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sB = smem + kOffB;
  uint8_t* sP = smem + kOffP;
  float* red_max = reinterpret_cast<float*>(smem + kOffRedMax);
  float* red_sum = reinterpret_cast<float*>(smem + kOffRedSum);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  const int seg_begin = __ldg(p.cta_seg + blockIdx.x);
  const int seg_end = __ldg(p.cta_seg + blockIdx.x + 1);
  const bool has_work = seg_begin < seg_end;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars[bFull + i], 1);
      mbar_init(&bars[bEmpty + i], 1);
    }
    mbar_init(&bars[bQFull], 1);
    mbar_init(&bars[bQEmpty], 1);
    mbar_init(&bars[bKrawFull], 1);
    mbar_init(&bars[bKpeFull], 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[bSFull + i], 1);
      mbar_init(&bars[bSFree + i], 4);
      mbar_init(&bars[bPFull + i], 4);
      mbar_init(&bars[bPvDone + i], 1);
    }
    mbar_init(&bars[bOFree], 4);
    mbar_init(&bars[bDrain], 1);
    mbar_init(&bars[bEpi], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_cache);
    tma_prefetch_desc(&tm_q);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  if (warp >= 2 && has_work) {
    // zero the query chunks (rows 24..31 stay zero: the TMA boxes are 24 rows) and build the rebuild B images:
    // K-step e holds rope_blocks[:, src_e : src_e + 16] as a K-major [64 x 16] no-swizzle operand
    // (8 x 16-byte core matrices: element (n, k) at (n / 8) * 256 + (k / 8) * 128 + (n % 8) * 16 + (k % 8) * 2).
    const int t = threadIdx.x - 64;
    uint4* q4 = reinterpret_cast<uint4*>(sQ);
    for (int i = t; i < kMaxQChunks * kQChunkBytes / 16; i += 128) q4[i] = make_uint4(0, 0, 0, 0);
    for (int e = 0; e < p.n_kst; ++e) {
      uint8_t* img = sB + e * kKstBytes;
      for (int idx = t; idx < 64 * 16; idx += 128) {
        const int n = idx >> 4, k = idx & 15;
        const __nv_bfloat16 v = p.rope_blocks[static_cast<long long>(n) * p.rope_ld + p.kst_src[e] + k];
        *reinterpret_cast<__nv_bfloat16*>(img + (n >> 3) * 256 + (k >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2) = v;
      }
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && has_work) {
      int fills = 0, qsegs = 0;
      bool ok = true;
      for (int s = seg_begin; s < seg_end && ok; ++s) {
        const SegmentInfo si = load_segment(p, s);
        if (!si.ok) {
          atomicCAS(p.err, 0, kErrBadSegment);
          continue;
        }
        if (qsegs > 0 && !(ok = mbar_wait(&bars[bQEmpty], (qsegs - 1) & 1, abort_flag, p.err, kErrTimeoutProducer)))
          break;
        mbar_arrive_expect_tx(&bars[bQFull], (p.n_k + kG) * 24 * 128);
        for (int c = 0; c < p.n_k + kG; ++c) tma_load_2d(sQ + c * kQChunkBytes, &tm_q, &bars[bQFull], c * 64, si.b * 24);
        ++qsegs;
        const int seq = __ldg(p.seq_lens + si.b);
        const int npages = (seq + p.page - 1) / p.page;
        const int32_t* bt = p.block_table + static_cast<long long>(si.b) * p.bt_stride;
        for (int tile = si.t0; tile < si.t1 && ok; ++tile) {
          int blk[8], row[8];
          for (int pc = 0; pc < p.n_pieces; ++pc) {
            const int tok0 = tile * kTile + pc * p.box_rows;
            const int pg = tok0 / p.page;
            row[pc] = tok0 - pg * p.page;
            blk[pc] = pg < npages ? __ldg(bt + pg) : p.num_blocks;   // past the request: an all-OOB (zero) box
          }
          for (int part = 0; part < p.n_kp + p.n_vp; ++part) {
            const int st = fills % kStages, rnd = fills / kStages;
            if (rnd > 0 && !(ok = mbar_wait(&bars[bEmpty + st], (rnd - 1) & 1, abort_flag, p.err,
                                            kErrTimeoutProducer)))
              break;
            int c0, halves;
            if (part < p.n_kp) {
              c0 = 128 * part;
              halves = (2 * part + 1 < p.n_k) ? 2 : 1;
            } else {
              const int j = part - p.n_kp;
              c0 = p.v_offset + 128 * j;
              halves = (128 * j + 64 < p.r_v) ? 2 : 1;
            }
            mbar_arrive_expect_tx(&bars[bFull + st], halves * kHalfBytes);
            uint8_t* dst = ring + st * kStageBytes;
            for (int h = 0; h < halves; ++h)
              for (int pc = 0; pc < p.n_pieces; ++pc)
                tma_load_3d(dst + h * kHalfBytes + pc * p.box_rows * 128, &tm_cache, &bars[bFull + st], c0 + 64 * h,
                            row[pc], blk[pc]);
            ++fills;
          }
        }
      }
      if (*abort_flag) {
        // let every copy this thread issued land before the CTA's shared memory goes away
        for (int k = max(0, fills - kStages); k < fills; ++k) mbar_wait_drain(&bars[bFull + k % kStages], (k / kStages) & 1);
        if (qsegs > 0) mbar_wait_drain(&bars[bQFull], (qsegs - 1) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0 && has_work) {
      constexpr uint32_t idS = idesc_bf16(128, 32, 0, 0);   // scores, K-major A and B
      constexpr uint32_t idK = idesc_bf16(128, 64, 0, 0);   // RoPE-key rebuild
      constexpr uint32_t idV = idesc_bf16(128, 32, 1, 1);   // O^T += V^T P, both MN-major
      const uint32_t ring_a = smem_u32(ring), q_a = smem_u32(sQ), b_a = smem_u32(sB), p_a = smem_u32(sP);
      int fills = 0, it = 0, qsegs = 0, segs = 0;
      bool ok = true;
      for (int s = seg_begin; s < seg_end && ok; ++s) {
        const SegmentInfo si = load_segment(p, s);
        if (!si.ok) continue;
        if (!(ok = mbar_wait(&bars[bQFull], qsegs & 1, abort_flag, p.err, kErrTimeoutMma))) break;
        ++qsegs;
        for (int tile = si.t0; tile < si.t1 && ok; ++tile) {
          const int sb = it & 1;
          if (it >= 2 && !(ok = mbar_wait(&bars[bSFree + sb], ((it >> 1) - 1) & 1, abort_flag, p.err, kErrTimeoutMma)))
            break;
          tc_fence_after();
          const uint32_t dS = tmem + 32 * sb;
          uint32_t acc = 0;
          for (int pp = 0; pp < p.n_kp; ++pp) {
            const int st = fills % kStages, rnd = fills / kStages;
            if (!(ok = mbar_wait(&bars[bFull + st], rnd & 1, abort_flag, p.err, kErrTimeoutMma))) break;
            tc_fence_after();
            const uint32_t base = ring_a + st * kStageBytes;
            for (int i = 0; i < 8; ++i) {
              const int col = 128 * pp + 16 * i;
              if (col >= 64 * p.n_k) break;
              const uint64_t a = smem_desc(base + (i >> 2) * kHalfBytes + (i & 3) * 32, 16, 1024, kSwizzle128);
              const uint64_t b = smem_desc(q_a + (col >> 6) * kQChunkBytes + (col & 63) * 2, 16, 1024, kSwizzle128);
              mma_ss(dS, a, b, idS, acc);
              acc = 1;
            }
            for (int e = 0; e < p.n_kst; ++e) {
              const int col = p.kst_col[e];
              if ((col >> 7) != pp) continue;
              const uint64_t a = smem_desc(base + ((col >> 6) & 1) * kHalfBytes + (col & 63) * 2, 16, 1024, kSwizzle128);
              const uint64_t b = smem_desc(b_a + e * kKstBytes, 128, 256, kSwizzleNone);
              mma_ss(tmem + kTmemK + 64 * p.kst_group[e], a, b, idK, p.kst_first[e] ? 0u : 1u);
            }
            mma_commit(&bars[bEmpty + st]);
            ++fills;
          }
          if (!ok) break;
          mma_commit(&bars[bKrawFull]);
          if (!(ok = mbar_wait(&bars[bKpeFull], it & 1, abort_flag, p.err, kErrTimeoutMma))) break;
          tc_fence_after();
          for (int g = 0; g < kG; ++g)
            for (int k = 0; k < 4; ++k) {
              const uint64_t b = smem_desc(q_a + (p.n_k + g) * kQChunkBytes + k * 32, 16, 1024, kSwizzle128);
              mma_ts(dS, tmem + kTmemK + 64 * g + 8 * k, b, idS, 1u);
            }
          mma_commit(&bars[bSFull + sb]);
          if (tile == si.t1 - 1) mma_commit(&bars[bQEmpty]);
          if (!(ok = mbar_wait(&bars[bPFull + sb], (it >> 1) & 1, abort_flag, p.err, kErrTimeoutMma))) break;
          if (tile == si.t0 && segs > 0 &&
              !(ok = mbar_wait(&bars[bOFree], (segs - 1) & 1, abort_flag, p.err, kErrTimeoutMma)))
            break;
          tc_fence_after();
          const uint32_t pbase = p_a + sb * kPBytes;
          for (int j = 0; j < p.n_vp; ++j) {
            const int st = fills % kStages, rnd = fills / kStages;
            if (!(ok = mbar_wait(&bars[bFull + st], rnd & 1, abort_flag, p.err, kErrTimeoutMma))) break;
            tc_fence_after();
            const uint32_t base = ring_a + st * kStageBytes;
            for (int k = 0; k < 8; ++k) {
              // A = V^T: MN-major SWIZZLE_128B, LBO = the second 64-feature half, SBO = 8 tokens (1 KB)
              const uint64_t a = smem_desc(base + k * 2048, kHalfBytes, 1024, kSwizzle128);
              // B = P [tokens x heads]: MN-major no swizzle, LBO = 8 tokens (512 B), SBO = 8 heads (128 B)
              const uint64_t b = smem_desc(pbase + k * 1024, 512, 128, kSwizzleNone);
              mma_ss(tmem + kTmemO + 32 * j, a, b, idV, (tile == si.t0 && k == 0) ? 0u : 1u);
            }
            mma_commit(&bars[bEmpty + st]);
            ++fills;
          }
          if (!ok) break;
          mma_commit(&bars[bPvDone + sb]);
          ++it;
        }
        ++segs;
      }
      if (*abort_flag) {
        mma_commit(&bars[bDrain]);
        mbar_wait_drain(&bars[bDrain], 0);
      }
    }
    __syncwarp();
  } else if (has_work) {
    // ------------------------------------------------------------------ epilogue: 128 threads = 128 TMEM lanes
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base, tK = tmem + lane_base + kTmemK, tO = tmem + lane_base + kTmemO;
    int it = 0, pv_seen = 0;
    bool ok = true;
    // every lane waits; the outcome is made warp-uniform so the .sync.aligned TMEM accesses stay convergent
    auto ewait = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool r = mbar_wait(bar, parity, abort_flag, p.err, kErrTimeoutEpilogue);
      return __all_sync(0xffffffffu, r);
    };
    uint32_t epi_phase = 0;
    auto epi_sync = [&]() -> bool {   // all 128 epilogue threads; shared-memory writes before it are visible after
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[bEpi]);
      const bool r = ewait(&bars[bEpi], epi_phase);
      epi_phase ^= 1u;
      return r;
    };
    auto wait_pv_until = [&](int k) -> bool {
      while (pv_seen <= k) {
        if (!ewait(&bars[bPvDone + (pv_seen & 1)], (pv_seen >> 1) & 1)) return false;
        ++pv_seen;
      }
      return true;
    };
    for (int s = seg_begin; s < seg_end && ok; ++s) {
      const SegmentInfo si = load_segment(p, s);
      if (!si.ok) continue;
      float m_run[kH], l_run[kH];
#pragma unroll
      for (int h = 0; h < kH; ++h) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.f;
      }
      for (int tile = si.t0; tile < si.t1 && ok; ++tile) {
        const int sb = it & 1;
        const int pos = tile * kTile + row;
        // ---- RoPE keys: BF16(gain * B_g c~), NeoX rotation at this token's position, BF16 operand
        uint4 cs[8];
        if (pos < p.max_pos) {
          const uint4* src = reinterpret_cast<const uint4*>(p.cos_sin + static_cast<long long>(pos) * kRot);
#pragma unroll
          for (int i = 0; i < 8; ++i) cs[i] = __ldg(src + i);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) cs[i] = make_uint4(0, 0, 0, 0);
        }
        if (!(ok = ewait(&bars[bKrawFull], it & 1))) break;
        tc_fence_after();
#pragma unroll 1
        for (int g = 0; g < kG; ++g) {
          uint32_t x[32], y[32], o[32];
          tmem_ld32(tK + 64 * g, x);
          tmem_ld32(tK + 64 * g + 32, y);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float x1a = bf16_round(__uint_as_float(x[2 * j])), x1b = bf16_round(__uint_as_float(x[2 * j + 1]));
            const float x2a = bf16_round(__uint_as_float(y[2 * j])), x2b = bf16_round(__uint_as_float(y[2 * j + 1]));
            const float ca = bf16_lane(cs, 2 * j), cb = bf16_lane(cs, 2 * j + 1);
            const float sa = bf16_lane(cs, 32 + 2 * j), sbv = bf16_lane(cs, 32 + 2 * j + 1);
            o[j] = pack_bf16(x1a * ca - x2a * sa, x1b * cb - x2b * sbv);
            o[16 + j] = pack_bf16(x2a * ca + x1a * sa, x2b * cb + x1b * sbv);
          }
          tmem_st32(tK + 64 * g, o);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[bKpeFull]);

        // ---- scores of this tile
        if (!(ok = ewait(&bars[bSFull + sb], (it >> 1) & 1))) break;
        tc_fence_after();
        uint32_t sr[32];
        tmem_ld32(tS + 32 * sb, sr);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[bSFree + sb]);
        const bool valid = pos < si.end;
        float z[kH];
#pragma unroll
        for (int h = 0; h < kH; ++h) z[h] = valid ? __uint_as_float(sr[h]) * p.scale_log2 : -INFINITY;
        float* rm = red_max + sb * 128;
#pragma unroll
        for (int h = 0; h < kH; ++h) {
          const float mh = warp_max(z[h]);
          if (lane == h) rm[ew * 32 + h] = mh;
        }
        if (!(ok = epi_sync())) break;
        float alpha[kH];
        bool rescale = false;
#pragma unroll
        for (int h = 0; h < kH; ++h) {
          const float mt = fmaxf(fmaxf(rm[h], rm[32 + h]), fmaxf(rm[64 + h], rm[96 + h]));
          alpha[h] = 1.f;
          if (m_run[h] == -INFINITY) {
            m_run[h] = mt;
          } else if (mt > m_run[h] + 8.f) {
            alpha[h] = exp2f(m_run[h] - mt);
            m_run[h] = mt;
            rescale = true;
          }
        }
        if (rescale) {   // uniform: every thread saw the same maxima
          if (!(ok = wait_pv_until(it - 1))) break;
          tc_fence_after();
          for (int j = 0; j < p.n_vp; ++j) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * j, o);
            tmem_ld_wait();
#pragma unroll
            for (int h = 0; h < kH; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
            tmem_st32(tO + 32 * j, o);
          }
          tmem_st_wait();
#pragma unroll
          for (int h = 0; h < kH; ++h) l_run[h] *= alpha[h];
        }
        if (it >= 2 && !(ok = wait_pv_until(it - 2))) break;   // P buffer sb is free again
        uint32_t w[16];
#pragma unroll
        for (int k = 0; k < 12; ++k) {
          const float pa = exp2f(z[2 * k] - m_run[2 * k]);
          const float pb = exp2f(z[2 * k + 1] - m_run[2 * k + 1]);
          l_run[2 * k] += pa;
          l_run[2 * k + 1] += pb;
          w[k] = pack_bf16(pa, pb);
        }
        w[12] = w[13] = w[14] = w[15] = 0u;
        uint8_t* prow = sP + sb * kPBytes + (row >> 3) * 512 + (row & 7) * 16;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(prow + c * 128) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[bPFull + sb]);
        ++it;
      }
      if (!ok) break;
      // ---- segment epilogue: normalised partial output and LSE
      if (!(ok = wait_pv_until(it - 1))) break;
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < kH; ++h) {
        const float sum = warp_sum(l_run[h]);
        if (lane == h) red_sum[ew * 32 + h] = sum;
      }
      if (!(ok = epi_sync())) break;
      float inv[kH];
#pragma unroll
      for (int h = 0; h < kH; ++h) {
        const float tot = red_sum[h] + red_sum[32 + h] + red_sum[64 + h] + red_sum[96 + h];
        inv[h] = 1.f / tot;
        if (row == h) p.part[static_cast<long long>(s) * p.part_ss + h * p.part_sh + p.r_v] =
            (m_run[h] + __log2f(tot)) * 0.69314718055994530942f;
      }
      for (int j = 0; j < p.n_vp; ++j) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * j, o);
        tmem_ld_wait();
        const int f = 128 * j + row;
        if (f < p.r_v) {
          float* dst = p.part + static_cast<long long>(s) * p.part_ss + f;
#pragma unroll
          for (int h = 0; h < kH; ++h) dst[h * p.part_sh] = __uint_as_float(o[h]) * inv[h];
        }
      }
      tc_fence_before();
      if (!(ok = epi_sync())) break;   // red_sum is reused by the next segment
      if (lane == 0) mbar_arrive(&bars[bOFree]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// host launch
// ---------------------------------------------------------------------------------------------------------------
int decode_smem_bytes() { return dec::kSmemBytes; }

cudaError_t launch_latent_decode(const CUtensorMap& tm_cache, const CUtensorMap& tm_q, const DecodeParams& p,
                                 int num_ctas, cudaStream_t stream) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(latent_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         dec::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  latent_decode_kernel<<<num_ctas, dec::kThreads, dec::kSmemBytes, stream>>>(tm_cache, tm_q, p);
  return cudaGetLastError();
}

}  // namespace belt
