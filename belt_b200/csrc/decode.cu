// Single-pass paged latent decode for sm_100a (tcgen05 + TMEM + TMA), split-KV over a persistent grid.
//
// Replaces the reference's Hopper CuTe kernel ``LatentDecodeSm90`` (plugins/vllm_lrkv/vllm_lrkv/cute_decode.py:90-484)
// with a Blackwell design. One CTA per SM walks the segments the schedule dealt it (cute_decode.py:571-598
// semantics, 128-token tiles). Twelve warps in three warpgroups; warpgroup 0 gives registers to the other two
// (setmaxnreg: 80 / 208 / 208 per thread, within the 3 x 168 the launch provides):
//
// * warp 0, TMA producer (lanes 0-15, one box per lane and stage, issued in one instruction): streams the cache
//   through a ring of stages, each `cps` 64-column chunks of 128 tokens, all SWIZZLE_128B. Two layouts:
//     - chunked (64-column-aligned row parts): one 5-D box {64 columns, 8 rows, n chunks, 8-row groups, 1 block} per
//       page (16 rows x 4 chunks = 8 KB at page 16), the 8-row groups landing as consecutive atoms of n KB;
//     - page (any 8-aligned layout): 3-D boxes of `page` rows x 64 columns, 2 chunks per stage.
//   Each lane reads its box's block id once per tile. Pages past the request are all-OOB boxes (zeros). Stage order is
//   software-pipelined across tiles: K(0), K(1), V(0), K(2), V(1), ... so that tile i's softmax runs while tile i+1's
//   key stages are scored and tile i's values stream in.
// * warp 1, tcgen05 issuer (one thread; descriptors advance only their low words), M = 128 tokens:
//     - scores S[tok, head] (N = 32: 24 heads; the last 8 columns are ignored) over the K part against the
//       block-diagonal query;
//     - the rebuilt RoPE keys gain * B_g c~_g: per group the 16-column K-steps holding its rr_g coordinates against
//       resident [64 x 16] images of the rope blocks (N = 64), into TMEM;
//     - after the rotation warps wrote the rotated BF16 keys back into TMEM, the RoPE score with A read from TMEM;
//     - O^T[latent, head] += V^T P per 128-latent block (A = the cache stage read MN-major, B = P from shared memory).
// * warp 2, query loader (lanes 0-15): a segment's block-diagonal query chunks, once the previous segment released them.
// * warp 3: idle.
// * warps 4-7, rotation: BF16(gain * B_g c~) -> NeoX rotation at each token's position in fp32 -> BF16 operand
//   (cute_decode.py:473-484), one TMEM lane (token) per thread; in packed fp32x2 arithmetic for narrow rows
//   (kPackedRot).
// * warps 8-11, softmax: masked online softmax in the exp2 domain; the running max of a head is raised only when a
//   tile exceeds it by more than 2^8 (a warp vote; the O rescale then waits for the previous P.V), P rounded to BF16
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
// A query chunk holds 24 rows of 128 bytes; the score MMA reads 32 rows (N = 32), the last 8 overlapping the next chunk:
// they only feed S columns 24..31, which nothing reads.
constexpr int kQChunkBytes = 24 * 128;
constexpr int kKstBytes = 64 * 16 * 2;          // [64 x 16] BF16 = 2 KB
constexpr int kPBytes = kTile * 32 * 2;         // [128 tokens x 32 heads] BF16 = 8 KB
constexpr int kThreads = 384;
constexpr int kRegsWg0 = 80, kRegsWork = 208;   // 80 + 2 * 208 <= 3 * 168 registers per SMSP
constexpr int kProducerLanes = 16;             // one TMA box per lane and stage (16 boxes of a 128-token stage)
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
constexpr int bImg = bSoft + 1;                // rebuild images written (4 rotation warps)
constexpr int kNumBars = 32;
static_assert(bImg < kNumBars, "barriers");
// red_max [2][4][32], red_sum [4][32], flags [2][4], per-head alpha / 1 / sum [32]
constexpr int kRedFloats = 2 * 4 * 32 + 4 * 32 + 2 * 4 + 32;
}  // namespace dec

bool decode_plan_smem(DecodeParams& p) {
  using namespace dec;
  auto up = [](int x, int a) { return (x + a - 1) / a * a; };
  const int q_bytes = up((p.n_k + kG) * kQChunkBytes + 1024, 1024);
  const int b_bytes = p.n_kst * kKstBytes;
  const int fixed = q_bytes + b_bytes + 2 * kPBytes + up(kRedFloats * 4, 128) + kNumBars * 8 + 16 + 1024;
  int stages = (kMaxSmem - fixed) / p.stage_bytes;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  p.stages = stages;
  p.off_q = stages * p.stage_bytes;
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

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
      "%7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
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

// kPackedRot: the rotation in packed fp32x2 arithmetic. It takes about a quarter fewer instructions, which pays
// where the rotation bounds the tile period (narrow rows: a c25 layer, 512 columns, runs 3 % faster) and costs
// 1-4 % where the softmax warps on the same schedulers bound it (1,024-column rows). The launcher picks it for rows of
// at most 4 + 4 chunks.
template <bool kChunked, bool kPackedRot>
__global__ void __launch_bounds__(dec::kThreads, 1)
    latent_decode_kernel(const __grid_constant__ DecodeMaps maps, const __grid_constant__ DecodeParams p) {
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
  unsigned long long* t_begin = reinterpret_cast<unsigned long long*>(tmem_slot + 2);   // the CTA's start (cta_ns)

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
    mbar_init(&bars[bImg], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < (kChunked ? 4 : 1); ++i) tma_prefetch_desc(&maps.cache[i]);
    tma_prefetch_desc(&maps.q);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the next kernel (the segment merge) may start launching; it waits for this grid before it reads the partials
  if (threadIdx.x == 0) allow_dependents_launch();

  if (warp < 4) {
   warpgroup_reg_dealloc<kRegsWg0>();
   if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (lanes 0-3)
    if (lane < kProducerLanes && has_work) {
      constexpr unsigned kLanes = (1u << kProducerLanes) - 1;
      int fills = 0;
      bool ok = true;
      // Where this lane's box of a tile comes from: chunked layout, tokens [box_rows lane, box_rows (lane + 1)) of the
      // tile (lanes < n_pieces); page layout, piece lane % n_pieces (of chunk lane / n_pieces). One block-table read
      // per lane and tile; pages past the request read as block num_blocks, all out of bounds (zeros).
      struct BoxPos {
        int blk, row;
      };
      auto box_pos = [&](const TileCursor& c) -> BoxPos {
        const int npages = (__ldg(p.seq_lens + c.si.b) + p.page - 1) / p.page;
        const int tok0 = c.tile * kTile + (kChunked ? lane : lane % p.n_pieces) * p.box_rows;
        const int pg = tok0 / p.page;
        BoxPos bp{p.num_blocks, tok0 - pg * p.page};
        if (pg < npages) bp.blk = __ldg(p.block_table + static_cast<long long>(c.si.b) * p.bt_stride + pg);
        return bp;
      };
      // one stage: chunks [chunk0, chunk0 + nch) (column col0 on), lane 0 waits for the slot and arms its barrier,
      // then every lane issues its box in the same instruction
      auto load_stage = [&](const BoxPos& bp, int col0, int chunk0, int nch) -> bool {
        const int st = fills % S;
        const int rnd = fills / S;
        bool got = true;
        if (lane == 0 && rnd > 0)
          got = mbar_wait(&bars[bEmpty + st], (rnd - 1) & 1, abort_flag, p.err, kErrTimeoutProducer);
        if (!__shfl_sync(kLanes, got ? 1 : 0, 0)) return false;
        if (lane == 0) mbar_arrive_expect_tx(&bars[bFull + st], nch * kTile * 128);
        __syncwarp(kLanes);
        uint8_t* dst = ring + st * p.stage_bytes;
        if constexpr (kChunked) {
          // 5-D box {64 columns, 8 rows, nch chunks, box_rows / 8 row groups, 1 block}: every 8-row group lands one atom
          // (nch chunks of 1 KB) after the previous one, so a stage's atoms are nch KB apart
          if (lane < p.n_pieces)
            tma_load_5d(dst + lane * (p.box_rows / 8) * nch * p.chunk_stride, &maps.cache[nch - 1], &bars[bFull + st], 0,
                        0, chunk0, bp.row / 8, bp.blk);
        } else if (lane < nch * p.n_pieces) {
          const int h = lane / p.n_pieces, pc = lane - h * p.n_pieces;
          tma_load_3d(dst + h * p.chunk_stride + pc * p.box_rows * 128, &maps.cache[0], &bars[bFull + st],
                      col0 + 64 * h, bp.row, bp.blk);
        }
        ++fills;
        return true;
      };
      TileCursor kc, vc;
      kc.begin(p, seg_begin, seg_end);
      vc.begin(p, seg_begin, seg_end);
      BoxPos pos_k{}, pos_v{};
      auto load_K = [&]() -> bool {
        pos_k = box_pos(kc);
        for (int k = 0; k < p.n_ks; ++k)
          if (!load_stage(pos_k, 64 * p.cps * k, p.cps * k, min(p.cps, p.n_k - p.cps * k))) return false;
        return true;
      };
      auto load_V = [&](const BoxPos& bp) -> bool {
        for (int k = 0; k < p.n_vs; ++k)
          if (!load_stage(bp, p.v_offset + 64 * p.cps * k, p.v_chunk0 + p.cps * k, min(p.cps, p.n_vc - p.cps * k)))
            return false;
        return true;
      };
      // stage order K(0), K(1), V(0), K(2), V(1), ...: V(i) reuses the box positions computed for K(i). (Taking V(i)
      // before K(i + 1) where tile i + 1 opens a segment was measured 4 % slower: the MMA issuer then idles while the
      // softmax finishes tile i, with the ring full of value stages.)
      if (kc.valid) {
        ok = load_K();
        pos_v = pos_k;
        kc.next(p);
      }
      while (ok && vc.valid) {
        const BoxPos cur_v = pos_v;
        if (kc.valid) {
          if (!(ok = load_K())) break;
          pos_v = pos_k;
          kc.next(p);
        }
        if (!(ok = load_V(cur_v))) break;
        vc.next(p);
      }
      if (lane == 0 && *abort_flag) {
        // let every copy issued land before the CTA's shared memory goes away
        for (int k = max(0, fills - S); k < fills; ++k) mbar_wait_drain(&bars[bFull + k % S], (k / S) & 1);
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
      // Descriptors (16-byte units): every operand's high word is fixed, a K step only moves the low word.
      constexpr uint32_t hiQ = desc_hi(1024, kSwizzle128);          // query chunks: 8 rows = 1 KB
      constexpr uint32_t hiImg = desc_hi(256, kSwizzleNone);        // rebuild images: 8 rows = 256 B
      constexpr uint32_t hiP = desc_hi(128, kSwizzleNone);          // P: 8 heads = 128 B
      const uint32_t loRing = desc_lo(ring_a, 16);                  // + stage, + chunk, + step * 2
      const uint32_t loRingV = desc_lo(ring_a, p.chunk_stride);     // V^T: LBO = the next 64-feature chunk
      const uint32_t loQ = desc_lo(q_a, 16);                        // + chunk * 192, + step * 2
      const uint32_t loImg = desc_lo(b_a, 128);                     // + e * 128
      const uint32_t loP = desc_lo(p_a, 512);                       // + buffer * 512, + step * 64
      const uint32_t stage16 = p.stage_bytes >> 4, chunk16 = p.chunk_stride >> 4;
      // chunked layout: a stage of nch chunks holds 8-token atoms of nch KB (the producer's boxes stack them densely);
      // page layout: chunks of 128 rows, atoms of 1 KB whatever the stage holds
      auto atom_of = [&](int nch) -> int { return kChunked ? nch * p.chunk_stride : p.atom_stride; };
      // key part of tile i: scores into S[i & 1] and the rebuilt RoPE keys
      auto mma_K = [&](const TileCursor& c, int i) -> bool {
        if (c.first()) {
          if (!wait(bQFull, qsegs & 1)) return false;
          ++qsegs;
        }
        const int sb = i & 1;
        if (i >= 2 && !wait(bSFree + sb, ((i >> 1) - 1) & 1)) return false;
        // The previous tile's RoPE-score MMAs read the rotated keys from the TMEM columns this tile's rebuild
        // overwrites: they were issued before, and tcgen05.mma operations of one thread execute in issue order, so
        // no wait (a wait here would drain the tensor pipe once per tile).
        tc_fence_after();
        const uint32_t dS = tmem + 32 * sb;
        for (int k = 0; k < p.n_ks; ++k) {
          int st;
          if (!full(st)) return false;
          const uint32_t a0 = loRing + st * stage16;
          const int c0 = p.cps * k, c1 = min(p.n_k, c0 + p.cps);
          const uint32_t hiSw = desc_hi(atom_of(c1 - c0), kSwizzle128);
          for (int cc = c0; cc < c1; ++cc) {
            const uint32_t ac = a0 + (cc - c0) * chunk16;
            const uint32_t bq = loQ + cc * (kQChunkBytes >> 4);
#pragma unroll
            for (int s16 = 0; s16 < 4; ++s16)
              mma_ss(dS, desc_of(ac + s16 * 2, hiSw), desc_of(bq + s16 * 2, hiQ), idS, (cc | s16) ? 1u : 0u);
          }
          // RoPE-key rebuild: every group's 16-column steps that fall in this stage's chunks (constant parameter offsets
          // only, so nothing but arithmetic sits between two MMA issues)
#pragma unroll
          for (int g = 0; g < kG; ++g) {
            const int ks0 = p.rope_ks0[g];
            const int lo = max(ks0, 4 * c0), hi = min(p.rope_ks1[g], 4 * c1 - 1);
            const uint32_t dK = tmem + kTmemK + 64 * g;
            uint64_t da = desc_of(a0 + (lo / 4 - c0) * chunk16 + (lo % 4) * 2, hiSw);
            uint64_t db = desc_of(loImg + (p.rope_e0[g] + lo - ks0) * (kKstBytes >> 4), hiImg);
            for (int ks = lo; ks <= hi; ++ks) {
              mma_ss(dK, da, db, idK, ks != ks0 ? 1u : 0u);
              // next 16 columns: +32 bytes along the swizzled row, or the start of the next chunk
              da += (ks % 4 == 3) ? chunk16 - 6 : 2;
              db += kKstBytes >> 4;
            }
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
        const uint32_t q0 = loQ + p.n_k * (kQChunkBytes >> 4);
#pragma unroll
        for (int g = 0; g < kG; ++g)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ts(dS, tmem + kTmemK + 64 * g + 8 * k, desc_of(q0 + g * (kQChunkBytes >> 4) + k * 2, hiQ), idS, 1u);
        mma_commit(&bars[bSFull + (i & 1)]);
        if (c.last()) mma_commit(&bars[bQEmpty]);   // the segment's query chunks are read for the last time
        return true;
      };
      // value part of tile i: O^T += V^T P, one 128-feature block (two chunks of a stage) at a time
      auto mma_V = [&](const TileCursor& c, int i) -> bool {
        const int pb = i & 1;
        if (!wait(bPFull + pb, (i >> 1) & 1)) return false;
        if (c.first()) {
          if (vsegs > 0 && !wait(bOFree, (vsegs - 1) & 1)) return false;
          ++vsegs;
        }
        tc_fence_after();
        const uint32_t p0 = loP + pb * (kPBytes >> 4);
        const uint32_t first = c.first() ? 1u : 0u;
        for (int k = 0; k < p.n_vs; ++k) {
          int st;
          if (!full(st)) return false;
          const uint32_t a0 = loRingV + st * stage16;
          const int nchv = min(p.cps, p.n_vc - p.cps * k);
          const uint32_t hiSw = desc_hi(atom_of(nchv), kSwizzle128);
          const uint32_t pv_step16 = (2 * atom_of(nchv)) >> 4;
          const int j0 = (p.cps * k) >> 1, j1 = min(p.n_vp, (p.cps * (k + 1)) >> 1);
          for (int j = j0; j < j1; ++j) {
            const uint32_t aj = a0 + (2 * j - p.cps * k) * chunk16;
            const uint32_t dO = tmem + kTmemO + 32 * j;
#pragma unroll
            for (int s16 = 0; s16 < 8; ++s16)
              // A = V^T (MN-major SW128, 16 tokens = 2 atoms per step), B = P (MN-major, 16 tokens = 1 KB per step)
              mma_ss(dO, desc_of(aj + s16 * pv_step16, hiSw), desc_of(p0 + s16 * (1024 >> 4), hiP), idV,
                     (first && s16 == 0) ? 0u : 1u);
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
      ok = wait(bImg, 0);   // the rotation warps' rebuild images
      if (ok && kc.valid) {
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
   } else if (warp == 2) {
    // ------------------------------------------------------------------ query loader (lanes 0-15): the segment's
    // block-diagonal query chunks, one per lane, as soon as the previous segment's last RoPE score released them
    if (lane < kProducerLanes && has_work) {
      constexpr unsigned kLanes = (1u << kProducerLanes) - 1;
      // the query comes from the kernel ahead of this one (the absorbed-query GEMM), which may still be running; every
      // global write of this kernel (the partials) comes after the query, so after this wait as well
      grid_dependency_wait();
      if (lane == 0) *t_begin = global_ns();
      int qsegs = 0;
      TileCursor c;
      c.begin(p, seg_begin, seg_end);
      for (; c.valid; c.next(p)) {
        if (!c.first()) continue;
        bool got = true;
        if (lane == 0 && qsegs > 0)   // waits a whole segment: sleep between polls
          got = mbar_wait_idle(&bars[bQEmpty], (qsegs - 1) & 1, abort_flag, p.err, kErrTimeoutProducer, 256);
        if (!__shfl_sync(kLanes, got ? 1 : 0, 0)) break;
        if (lane == 0) mbar_arrive_expect_tx(&bars[bQFull], (p.n_k + kG) * kQChunkBytes);
        __syncwarp(kLanes);
        if (lane < p.n_k + kG) tma_load_2d(sQ + lane * kQChunkBytes, &maps.q, &bars[bQFull], lane * 64, c.si.b * kH);
        ++qsegs;
      }
      if (lane == 0 && *abort_flag && qsegs > 0) mbar_wait_drain(&bars[bQFull], (qsegs - 1) & 1);
    }
    __syncwarp();
   }
   // warp 3: no role
  } else if (warp < 8) {
    // ------------------------------------------------------------------ rotation warps: RoPE keys
    warpgroup_reg_alloc<kRegsWork>();
    if (has_work) {
      {
        // rebuild B images: K-step e holds rope_blocks[:, src_e : src_e + 16] as a K-major [64 x 16] no-swizzle
        // operand (8 x 16-byte core matrices: element (n, k) at (n / 8) * 256 + (k / 8) * 128 + (n % 8) * 16 +
        // (k % 8) * 2). 16-byte pieces (K-step, row, 8-column half), all loads issued before the stores; built while
        // the first stages stream in, the MMA issuer waits for bImg before its first rebuild.
        const int t = threadIdx.x - 128;
        uint4 v[kDecodeMaxKsteps];
#pragma unroll
        for (int e = 0; e < kDecodeMaxKsteps; ++e)
          if (e < p.n_kst) {
            const int n = t >> 1, h = t & 1;
            v[e] = __ldg(reinterpret_cast<const uint4*>(p.rope_blocks + static_cast<long long>(n) * p.rope_ld +
                                                         p.kst_src[e] + 8 * h));
          }
#pragma unroll
        for (int e = 0; e < kDecodeMaxKsteps; ++e)
          if (e < p.n_kst) {
            const int n = t >> 1, h = t & 1;
            *reinterpret_cast<uint4*>(sB + e * kKstBytes + (n >> 3) * 256 + h * 128 + (n & 7) * 16) = v[e];
          }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[bImg]);
      }
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
          if constexpr (kPackedRot) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // channel pairs as packed fp32x2 (low element first): x1 = bf16(x[2j], x[2j + 1]), x2 = bf16(y[2j], ..)
              const uint32_t xw = pack_bf16(__uint_as_float(x[2 * j]), __uint_as_float(x[2 * j + 1]));
              const uint32_t yw = pack_bf16(__uint_as_float(y[2 * j]), __uint_as_float(y[2 * j + 1]));
              const uint4 cq = cs[j >> 2], sq = cs[4 + (j >> 2)];
              const uint32_t cw = (j & 3) == 0 ? cq.x : (j & 3) == 1 ? cq.y : (j & 3) == 2 ? cq.z : cq.w;
              const uint32_t sw = (j & 3) == 0 ? sq.x : (j & 3) == 1 ? sq.y : (j & 3) == 2 ? sq.z : sq.w;
              auto wide = [](uint32_t w) -> unsigned long long {   // bf16x2 -> f32x2
                return static_cast<unsigned long long>(w << 16) |
                       (static_cast<unsigned long long>(w & 0xFFFF0000u) << 32);
              };
              const unsigned long long x1 = wide(xw), x2 = wide(yw), nx2 = wide(yw ^ 0x80008000u), c2 = wide(cw),
                                       s2 = wide(sw);
              unsigned long long t1, t2, r1, r2;
              asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(t1) : "l"(nx2), "l"(s2));
              asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r1) : "l"(x1), "l"(c2), "l"(t1));   // x1 cos - x2 sin
              asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(t2) : "l"(x1), "l"(s2));
              asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r2) : "l"(x2), "l"(c2), "l"(t2));    // x2 cos + x1 sin
              o[j] = pack_bf16(__uint_as_float(static_cast<uint32_t>(r1)),
                               __uint_as_float(static_cast<uint32_t>(r1 >> 32)));
              o[16 + j] = pack_bf16(__uint_as_float(static_cast<uint32_t>(r2)),
                                    __uint_as_float(static_cast<uint32_t>(r2 >> 32)));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float x1a = bf16_round(__uint_as_float(x[2 * j])), x1b = bf16_round(__uint_as_float(x[2 * j + 1]));
              const float x2a = bf16_round(__uint_as_float(y[2 * j])), x2b = bf16_round(__uint_as_float(y[2 * j + 1]));
              const float ca = bf16_lane(cs, 2 * j), cb = bf16_lane(cs, 2 * j + 1);
              const float sa = bf16_lane(cs, 32 + 2 * j), sbv = bf16_lane(cs, 32 + 2 * j + 1);
              o[j] = pack_bf16(x1a * ca - x2a * sa, x1b * cb - x2b * sbv);
              o[16 + j] = pack_bf16(x2a * ca + x1a * sa, x2b * cb + x1b * sbv);
            }
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
  // the CTA's time from its predecessor's completion to here, for the next step's balanced split
  if (threadIdx.x == 0 && p.cta_ns && has_work && !*abort_flag) atomicAdd(p.cta_ns + blockIdx.x, global_ns() - *t_begin);
}

// ---------------------------------------------------------------------------------------------------------------
// host launch
// ---------------------------------------------------------------------------------------------------------------
cudaError_t launch_latent_decode(const DecodeMaps& maps, const DecodeParams& p, int num_ctas, cudaStream_t stream) {
  static bool attr_done[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const bool packed = p.n_k <= 4 && p.n_vc <= 4;   // narrow rows: the rotation bounds the tile period
  const int m = (p.chunked ? 1 : 0) + (packed ? 2 : 0);
  auto kernel = packed ? (p.chunked ? latent_decode_kernel<true, true> : latent_decode_kernel<false, true>)
                       : (p.chunked ? latent_decode_kernel<true, false> : latent_decode_kernel<false, false>);
  if (dev >= 0 && dev < 64 && !attr_done[m][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::kMaxSmem);
    if (e != cudaSuccess) return e;
    attr_done[m][dev] = true;
  }
  cudaError_t e = launch_after(kernel, dim3(num_ctas), dim3(dec::kThreads), p.smem_bytes, stream, maps, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace belt
