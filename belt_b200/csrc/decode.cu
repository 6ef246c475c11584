// Single-pass paged latent decode for sm_100a (tcgen05 + TMEM + TMA), split-KV over a persistent grid.
//
// Replaces the reference's Hopper CuTe kernel ``LatentDecodeSm90`` (plugins/vllm_lrkv/vllm_lrkv/cute_decode.py:90-484)
// with a Blackwell design. One CTA per SM walks the segments the schedule dealt it (cute_decode.py:571-598
// semantics, 128-token tiles). Twelve warps in three warpgroups; warpgroup 0 gives registers to the other two
// (setmaxnreg: 80 / 208 / 208 per thread, within the 3 x 168 the launch provides):
//
// * warp 0, TMA producer: streams the cache through a ring of 32 KB stages = [128 tokens x 128 features] as two
//   SWIZZLE_128B halves of [128 x 64]. Pages of 16..128 tokens are fetched as boxes of `page` rows through a 3-D tensor
//   map over the (possibly strided) [blocks, page, W] cache view; pages past the request are all-OOB boxes (zeros).
//   Stage order is software-pipelined across tiles: K(0), K(1), V(0), K(2), V(1), ... so that tile i's softmax runs
//   while tile i+1's key stages are scored and tile i's value stages stream in.
// * warp 1, tcgen05 issuer (one thread), M = 128 tokens:
//     - scores S[tok, head] (N = 32: 24 heads; the last 8 columns are ignored) over the K part against the
//       block-diagonal query;
//     - the rebuilt RoPE keys gain * B_g c~_g: per group the 16-column K-steps holding its rr_g coordinates against
//       resident [64 x 16] images of the rope blocks (N = 64), into TMEM;
//     - after the rotation warps wrote the rotated BF16 keys back into TMEM, the RoPE score with A read from TMEM;
//     - O^T[latent, head] += V^T P per 128-latent block (A = the cache stage read MN-major, B = P from shared memory).
// * warps 2-3: idle.
// * warps 4-7, rotation: BF16(gain * B_g c~) -> NeoX rotation at each token's position in fp32 -> BF16 operand
//   (cute_decode.py:473-484), one TMEM lane (token) per thread.
// * warps 8-11, softmax: masked online softmax in the exp2 domain; the running max of a head is raised only when a tile
//   exceeds it by more than 2^8 (a warp vote; the O rescale then waits for the previous P.V), P rounded to BF16
//   (cute_decode.py:408); per segment the normalised partial output and its natural-log LSE (cute_decode.py:435-455).
//
// TMEM columns: [0, 64) two S buffers, [64, 320) the four groups' rebuilt keys (fp32; the rotated BF16 keys are packed
// into the first 32 columns of each group's range), [320, 320 + 32 * n_vp) the O^T blocks.
//
// Every wait is bounded (common.cuh): a logic error records a code in the device error word and the CTA drains what
// it issued, frees its tensor memory and exits.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace dec {
constexpr int kTile = 128;
constexpr int kMaxStages = 5;
constexpr int kHalfBytes = kTile * 64 * 2;      // [128 x 64] BF16 = 16 KB
constexpr int kStageBytes = 2 * kHalfBytes;     // 32 KB
// A query chunk holds 24 rows of 128 bytes; the score MMA reads 32 rows (N = 32), the last 8 overlapping the next chunk:
// they only feed S columns 24..31, which nothing reads.
constexpr int kQChunkBytes = 24 * 128;
constexpr int kKstBytes = 64 * 16 * 2;          // [64 x 16] BF16 = 2 KB
constexpr int kPBytes = kTile * 32 * 2;         // [128 tokens x 32 heads] BF16 = 8 KB
constexpr int kThreads = 384;
constexpr int kRegsWg0 = 80, kRegsWork = 208;   // 80 + 2 * 208 <= 3 * 168 registers per SMSP
constexpr int kTmemCols = 512;
constexpr int kTmemK = 64;
constexpr int kTmemO = 320;
constexpr int kMaxSmem = 232448;

// barrier indices
constexpr int bFull = 0;                       // [kMaxStages]
constexpr int bEmpty = bFull + kMaxStages;     // [kMaxStages]
constexpr int bQFull = bEmpty + kMaxStages;
constexpr int bQEmpty = bQFull + 1;
constexpr int bKrawFull = bQEmpty + 1;
constexpr int bKpeFull = bKrawFull + 1;
constexpr int bSFull = bKpeFull + 1;           // [2]
constexpr int bSFree = bSFull + 2;             // [2]
constexpr int bPFull = bSFree + 2;             // [2]
constexpr int bPvDone = bPFull + 2;            // [2]
constexpr int bOFree = bPvDone + 2;
constexpr int bDrain = bOFree + 1;
constexpr int bSoft = bDrain + 1;              // softmax group barrier (4 warps)
constexpr int kNumBars = 32;
static_assert(bSoft < kNumBars, "barriers");
// red_max [2][4][32], red_sum [4][32], flags [2][4], per-head alpha / 1 / sum [32]
constexpr int kRedFloats = 2 * 4 * 32 + 4 * 32 + 2 * 4 + 32;
}  // namespace dec

bool decode_plan_smem(DecodeParams& p) {
  using namespace dec;
  auto up = [](int x, int a) { return (x + a - 1) / a * a; };
  const int q_bytes = up((p.n_k + kG) * kQChunkBytes + 1024, 1024);
  const int b_bytes = p.n_kst * kKstBytes;
  const int fixed = q_bytes + b_bytes + 2 * kPBytes + up(kRedFloats * 4, 128) + kNumBars * 8 + 16 + 1024;
  int stages = (kMaxSmem - fixed) / kStageBytes;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  p.stages = stages;
  p.off_q = stages * kStageBytes;
  p.off_b = p.off_q + q_bytes;
  p.off_p = p.off_b + b_bytes;
  p.off_red = p.off_p + 2 * kPBytes;
  p.off_bars = p.off_red + up(kRedFloats * 4, 128);
  p.smem_bytes = p.off_bars + kNumBars * 8 + 16 + 1024;
  return p.smem_bytes <= kMaxSmem;
}

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
  const int seq = si.ok ? __ldg(p.seq_lens + si.b) : 0;
  si.ok = si.ok && (si.t1 - 1) * dec::kTile < seq;
  si.end = min(si.t1 * dec::kTile, seq);
  return si;
}

// Walks this CTA's tiles in order, segment by segment (every role iterates the same sequence).
struct TileCursor {
  int s, s_end, tile;
  SegmentInfo si;
  bool valid;
  __device__ void begin(const DecodeParams& p, int s_begin, int s_stop) {
    s = s_begin - 1;
    s_end = s_stop;
    advance(p);
  }
  __device__ void advance(const DecodeParams& p) {
    valid = false;
    while (++s < s_end) {
      si = load_segment(p, s);
      if (si.ok) {
        tile = si.t0;
        valid = true;
        return;
      }
    }
  }
  __device__ void next(const DecodeParams& p) {
    if (++tile >= si.t1) advance(p);
  }
  __device__ bool first() const { return tile == si.t0; }
  __device__ bool last() const { return tile == si.t1 - 1; }
};

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
  uint8_t* ring = smem;
  uint8_t* sQ = smem + p.off_q;
  uint8_t* sB = smem + p.off_b;
  uint8_t* sP = smem + p.off_p;
  float* red_max = reinterpret_cast<float*>(smem + p.off_red);   // [2][4][32]
  float* red_sum = red_max + 2 * 4 * 32;                          // [4][32]
  int* flags = reinterpret_cast<int*>(red_sum + 4 * 32);          // [2][4]
  float* head_s = reinterpret_cast<float*>(flags + 8);            // [32] per-head alpha or 1 / sum
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int seg_begin = __ldg(p.cta_seg + blockIdx.x);
  const int seg_end = __ldg(p.cta_seg + blockIdx.x + 1);
  const bool has_work = seg_begin < seg_end;
  const int S = p.stages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
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
    mbar_init(&bars[bSoft], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_cache);
    tma_prefetch_desc(&tm_q);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  if (warp >= 4 && warp < 8 && has_work) {
    // rebuild B images: K-step e holds rope_blocks[:, src_e : src_e + 16] as a K-major [64 x 16] no-swizzle operand
    // (8 x 16-byte core matrices: element (n, k) at (n / 8) * 256 + (k / 8) * 128 + (n % 8) * 16 + (k % 8) * 2)
    const int t = threadIdx.x - 128;
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

  if (warp < 4) {
   warpgroup_reg_dealloc<kRegsWg0>();
   if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && has_work) {
      int fills = 0, qsegs = 0;
      bool ok = true;
      auto acquire = [&](int& st) -> bool {
        st = fills % S;
        const int rnd = fills / S;
        return rnd == 0 || mbar_wait(&bars[bEmpty + st], (rnd - 1) & 1, abort_flag, p.err, kErrTimeoutProducer);
      };
      auto tile_blocks = [&](const TileCursor& c, int* blk, int* row) {
        const int seq = __ldg(p.seq_lens + c.si.b);
        const int npages = (seq + p.page - 1) / p.page;
        const int32_t* bt = p.block_table + static_cast<long long>(c.si.b) * p.bt_stride;
        for (int pc = 0; pc < p.n_pieces; ++pc) {
          const int tok0 = c.tile * kTile + pc * p.box_rows;
          const int pg = tok0 / p.page;
          row[pc] = tok0 - pg * p.page;
          blk[pc] = pg < npages ? __ldg(bt + pg) : p.num_blocks;   // past the request: an all-OOB (zero) box
        }
      };
      auto load_stage = [&](int c0, int halves, const int* blk, const int* row) -> bool {
        int st;
        if (!acquire(st)) return false;
        mbar_arrive_expect_tx(&bars[bFull + st], halves * kHalfBytes);
        uint8_t* dst = ring + st * kStageBytes;
        for (int h = 0; h < halves; ++h)
          for (int pc = 0; pc < p.n_pieces; ++pc)
            tma_load_3d(dst + h * kHalfBytes + pc * p.box_rows * 128, &tm_cache, &bars[bFull + st], c0 + 64 * h,
                        row[pc], blk[pc]);
        ++fills;
        return true;
      };
      auto load_K = [&](const TileCursor& c) -> bool {
        if (c.first()) {
          if (qsegs > 0 && !mbar_wait(&bars[bQEmpty], (qsegs - 1) & 1, abort_flag, p.err, kErrTimeoutProducer))
            return false;
          mbar_arrive_expect_tx(&bars[bQFull], (p.n_k + kG) * kQChunkBytes);
          for (int ch = 0; ch < p.n_k + kG; ++ch)
            tma_load_2d(sQ + ch * kQChunkBytes, &tm_q, &bars[bQFull], ch * 64, c.si.b * kH);
          ++qsegs;
        }
        int blk[8], row[8];
        tile_blocks(c, blk, row);
        for (int pp = 0; pp < p.n_kp; ++pp)
          if (!load_stage(128 * pp, (2 * pp + 1 < p.n_k) ? 2 : 1, blk, row)) return false;
        return true;
      };
      auto load_V = [&](const TileCursor& c) -> bool {
        int blk[8], row[8];
        tile_blocks(c, blk, row);
        for (int j = 0; j < p.n_vp; ++j)
          if (!load_stage(p.v_offset + 128 * j, (128 * j + 64 < p.r_v) ? 2 : 1, blk, row)) return false;
        return true;
      };
      TileCursor kc, vc;
      kc.begin(p, seg_begin, seg_end);
      vc.begin(p, seg_begin, seg_end);
      if (kc.valid) {
        ok = load_K(kc);
        kc.next(p);
      }
      while (ok && vc.valid) {
        if (kc.valid) {
          if (!(ok = load_K(kc))) break;
          kc.next(p);
        }
        if (!(ok = load_V(vc))) break;
        vc.next(p);
      }
      if (*abort_flag) {
        // let every copy this thread issued land before the CTA's shared memory goes away
        for (int k = max(0, fills - S); k < fills; ++k) mbar_wait_drain(&bars[bFull + k % S], (k / S) & 1);
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
      int fills = 0, qsegs = 0, vsegs = 0;
      bool ok = true;
      auto wait = [&](int bar, uint32_t parity) -> bool {
        return mbar_wait(&bars[bar], parity, abort_flag, p.err, kErrTimeoutMma);
      };
      auto full = [&](int& st) -> bool {
        st = fills % S;
        if (!wait(bFull + st, (fills / S) & 1)) return false;
        tc_fence_after();
        return true;
      };
      // key part of tile i: scores into S[i & 1] and the rebuilt RoPE keys
      auto mma_K = [&](const TileCursor& c, int i) -> bool {
        if (c.first()) {
          if (!wait(bQFull, qsegs & 1)) return false;
          ++qsegs;
        }
        const int sb = i & 1;
        if (i >= 2 && !wait(bSFree + sb, ((i >> 1) - 1) & 1)) return false;
        // the previous tile's RoPE-score MMAs read the rotated keys from the TMEM columns the rebuild overwrites
        if (i >= 1 && !wait(bSFull + ((i - 1) & 1), ((i - 1) >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t dS = tmem + 32 * sb;
        uint32_t acc = 0;
        for (int pp = 0; pp < p.n_kp; ++pp) {
          int st;
          if (!full(st)) return false;
          const uint32_t base = ring_a + st * kStageBytes;
          for (int i16 = 0; i16 < 8; ++i16) {
            const int col = 128 * pp + 16 * i16;
            if (col >= 64 * p.n_k) break;
            const uint64_t a = smem_desc(base + (i16 >> 2) * kHalfBytes + (i16 & 3) * 32, 16, 1024, kSwizzle128);
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
        mma_commit(&bars[bKrawFull]);
        return true;
      };
      // RoPE score of tile i once the rotation warps stored its keys
      auto mma_rope = [&](const TileCursor& c, int i) -> bool {
        if (!wait(bKpeFull, i & 1)) return false;
        tc_fence_after();
        const uint32_t dS = tmem + 32 * (i & 1);
        for (int g = 0; g < kG; ++g)
          for (int k = 0; k < 4; ++k) {
            const uint64_t b = smem_desc(q_a + (p.n_k + g) * kQChunkBytes + k * 32, 16, 1024, kSwizzle128);
            mma_ts(dS, tmem + kTmemK + 64 * g + 8 * k, b, idS, 1u);
          }
        mma_commit(&bars[bSFull + (i & 1)]);
        if (c.last()) mma_commit(&bars[bQEmpty]);   // the segment's query chunks are read for the last time
        return true;
      };
      // value part of tile i: O^T += V^T P
      auto mma_V = [&](const TileCursor& c, int i) -> bool {
        const int pb = i & 1;
        if (!wait(bPFull + pb, (i >> 1) & 1)) return false;
        if (c.first()) {
          if (vsegs > 0 && !wait(bOFree, (vsegs - 1) & 1)) return false;
          ++vsegs;
        }
        tc_fence_after();
        const uint32_t pbase = p_a + pb * kPBytes;
        for (int j = 0; j < p.n_vp; ++j) {
          int st;
          if (!full(st)) return false;
          const uint32_t base = ring_a + st * kStageBytes;
          for (int k = 0; k < 8; ++k) {
            // A = V^T: MN-major SWIZZLE_128B, LBO = the second 64-feature half, SBO = 8 tokens (1 KB)
            const uint64_t a = smem_desc(base + k * 2048, kHalfBytes, 1024, kSwizzle128);
            // B = P [tokens x heads]: MN-major no swizzle, LBO = 8 tokens (512 B), SBO = 8 heads (128 B)
            const uint64_t b = smem_desc(pbase + k * 1024, 512, 128, kSwizzleNone);
            mma_ss(tmem + kTmemO + 32 * j, a, b, idV, (c.first() && k == 0) ? 0u : 1u);
          }
          mma_commit(&bars[bEmpty + st]);
          ++fills;
        }
        mma_commit(&bars[bPvDone + pb]);
        return true;
      };
      TileCursor kc, vc;
      kc.begin(p, seg_begin, seg_end);
      vc.begin(p, seg_begin, seg_end);
      if (kc.valid) {
        ok = mma_K(kc, 0) && mma_rope(kc, 0);
        kc.next(p);
      }
      for (int v = 0; ok && vc.valid; ++v) {
        const bool more = kc.valid;
        if (more && !(ok = mma_K(kc, v + 1))) break;
        if (!(ok = mma_V(vc, v))) break;
        if (more) {
          if (!(ok = mma_rope(kc, v + 1))) break;
          kc.next(p);
        }
        vc.next(p);
      }
      if (*abort_flag) {
        mma_commit(&bars[bDrain]);
        mbar_wait_drain(&bars[bDrain], 0);
      }
    }
    __syncwarp();
   }
   // warps 2-3: no role
  } else if (warp < 8) {
    // ------------------------------------------------------------------ rotation warps: RoPE keys
    warpgroup_reg_alloc<kRegsWork>();
    if (has_work) {
      const int quad = warp & 3;
      const int row = quad * 32 + lane;
      const uint32_t tK = tmem + (static_cast<uint32_t>(quad * 32) << 16) + kTmemK;
      TileCursor c;
      c.begin(p, seg_begin, seg_end);
      for (int i = 0; c.valid; ++i, c.next(p)) {
        const int pos = c.tile * kTile + row;
        uint4 cs[8];
        if (pos < p.max_pos) {
          const uint4* src = reinterpret_cast<const uint4*>(p.cos_sin + static_cast<long long>(pos) * kRot);
#pragma unroll
          for (int k = 0; k < 8; ++k) cs[k] = __ldg(src + k);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) cs[k] = make_uint4(0, 0, 0, 0);
        }
        const bool got = mbar_wait(&bars[bKrawFull], i & 1, abort_flag, p.err, kErrTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, got)) break;
        tc_fence_after();
#pragma unroll 1
        for (int g = 0; g < kG; ++g) {
          // all 64 fp32 channels are read before the packed BF16 keys overwrite the group's first 32 columns
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
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    warpgroup_reg_alloc<kRegsWork>();
    if (has_work) {
      const int sw = warp - 8;
      const int quad = warp & 3;
      const int row = quad * 32 + lane;
      const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
      const uint32_t tS = tmem + lane_base, tO = tmem + lane_base + kTmemO;
      int pv_seen = 0;
      uint32_t soft_phase = 0;
      bool ok = true;
      // every lane waits; the outcome is made warp-uniform so the .sync.aligned TMEM accesses stay convergent
      auto ewait = [&](int bar, uint32_t parity) -> bool {
        const bool r = mbar_wait(&bars[bar], parity, abort_flag, p.err, kErrTimeoutEpilogue);
        return __all_sync(0xffffffffu, r);
      };
      auto soft_sync = [&]() -> bool {   // the 4 softmax warps; shared-memory writes before it are visible after
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[bSoft]);
        const bool r = ewait(bSoft, soft_phase);
        soft_phase ^= 1u;
        return r;
      };
      auto wait_pv_until = [&](int k) -> bool {
        while (pv_seen <= k) {
          if (!ewait(bPvDone + (pv_seen & 1), (pv_seen >> 1) & 1)) return false;
          ++pv_seen;
        }
        return true;
      };
      float m_run[kH], l_run[kH];
      TileCursor c;
      c.begin(p, seg_begin, seg_end);
      for (int i = 0; ok && c.valid; ++i, c.next(p)) {
        if (c.first()) {
#pragma unroll
          for (int h = 0; h < kH; ++h) {
            m_run[h] = -INFINITY;
            l_run[h] = 0.f;
          }
        }
        const int sb = i & 1;
        const int pos = c.tile * kTile + row;
        if (!(ok = ewait(bSFull + sb, (i >> 1) & 1))) break;
        tc_fence_after();
        float z[kH];
        {
          uint32_t s16[16], s8[8];
          tmem_ld16(tS + 32 * sb, s16);
          tmem_ld8(tS + 32 * sb + 16, s8);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[bSFree + sb]);
          const bool valid = pos < c.si.end;
#pragma unroll
          for (int h = 0; h < 16; ++h) z[h] = valid ? __uint_as_float(s16[h]) * p.scale_log2 : -INFINITY;
#pragma unroll
          for (int h = 0; h < 8; ++h) z[16 + h] = valid ? __uint_as_float(s8[h]) * p.scale_log2 : -INFINITY;
        }
        bool need = false;
#pragma unroll
        for (int h = 0; h < kH; ++h) need |= z[h] > m_run[h] + 8.f;
        need = __any_sync(0xffffffffu, need);
        if (lane == 0) flags[sb * 4 + sw] = need ? 1 : 0;
        if (!(ok = soft_sync())) break;
        if (flags[sb * 4] | flags[sb * 4 + 1] | flags[sb * 4 + 2] | flags[sb * 4 + 3]) {
          // some head's tile max exceeds its running max by more than 2^8: reduce the tile's maxima
          float* rm = red_max + sb * 128;
#pragma unroll
          for (int h = 0; h < kH; ++h) {
            const float mh = warp_max(z[h]);
            if (lane == h) rm[sw * 32 + h] = mh;
          }
          if (!(ok = soft_sync())) break;
          bool rescale = false;
#pragma unroll
          for (int h = 0; h < kH; ++h) {
            const float mt = fmaxf(fmaxf(rm[h], rm[32 + h]), fmaxf(rm[64 + h], rm[96 + h]));
            float alpha = 1.f;
            if (mt > m_run[h] + 8.f) {
              if (m_run[h] != -INFINITY) {
                alpha = exp2f(m_run[h] - mt);
                rescale = true;
              }
              m_run[h] = mt;
            }
            l_run[h] *= alpha;
            if (sw == 0 && lane == h) head_s[h] = alpha;   // the same value in every thread
          }
          if (rescale) {   // uniform: every thread saw the same maxima
            if (!(ok = soft_sync())) break;                // head_s written
            if (!(ok = wait_pv_until(i - 1))) break;
            tc_fence_after();
            for (int j = 0; j < p.n_vp; ++j) {
              uint32_t o[32];
              tmem_ld32(tO + 32 * j, o);
              tmem_ld_wait();
#pragma unroll
              for (int h = 0; h < kH; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * head_s[h]);
              tmem_st32(tO + 32 * j, o);
            }
            tmem_st_wait();
          }
        }
        if (i >= 2 && !(ok = wait_pv_until(i - 2))) break;   // P buffer sb is free again
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
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(prow + k * 128) = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[bPFull + sb]);

        if (c.last()) {
          // ---- segment epilogue: normalised partial output and LSE
          const int s = c.s;
          if (!(ok = wait_pv_until(i))) break;
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < kH; ++h) {
            const float sum = warp_sum(l_run[h]);
            if (lane == h) red_sum[sw * 32 + h] = sum;
          }
          if (!(ok = soft_sync())) break;
          if (sw == 0 && lane < kH) {
            const float tot = red_sum[lane] + red_sum[32 + lane] + red_sum[64 + lane] + red_sum[96 + lane];
            head_s[lane] = 1.f / tot;
          }
#pragma unroll
          for (int h = 0; h < kH; ++h) {
            if (row == h) {
              const float tot = red_sum[h] + red_sum[32 + h] + red_sum[64 + h] + red_sum[96 + h];
              p.part[static_cast<long long>(s) * p.part_ss + h * p.part_sh + p.r_v] =
                  (m_run[h] + __log2f(tot)) * 0.69314718055994530942f;
            }
          }
          if (!(ok = soft_sync())) break;   // head_s = 1 / sum
          for (int j = 0; j < p.n_vp; ++j) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * j, o);
            tmem_ld_wait();
            const int f = 128 * j + row;
            if (f < p.r_v) {
              float* dst = p.part + static_cast<long long>(s) * p.part_ss + f;
#pragma unroll
              for (int h = 0; h < kH; ++h) dst[h * p.part_sh] = __uint_as_float(o[h]) * head_s[h];
            }
          }
          tc_fence_before();
          if (!(ok = soft_sync())) break;   // red_sum is reused by the next segment
          if (lane == 0) mbar_arrive(&bars[bOFree]);
        }
      }
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
cudaError_t launch_latent_decode(const CUtensorMap& tm_cache, const CUtensorMap& tm_q, const DecodeParams& p,
                                 int num_ctas, cudaStream_t stream) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(latent_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         dec::kMaxSmem);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  latent_decode_kernel<<<num_ctas, dec::kThreads, p.smem_bytes, stream>>>(tm_cache, tm_q, p);
  return cudaGetLastError();
}

}  // namespace belt
