// Single-pass paged latent decode for sm_100a (tcgen05 + TMEM + TMA), split-KV over a persistent grid.
//
// Replaces the reference's Hopper CuTe kernel ``LatentDecodeSm90`` (plugins/vllm_lrkv/vllm_lrkv/cute_decode.py:90-484)
// with a Blackwell design. One CTA per SM walks the segments the schedule dealt it (cute_decode.py:571-598
// semantics, 128-token tiles). Twelve warps in three warpgroups; warpgroup 0 gives registers to the other two
// (setmaxnreg: 104 / 200 / 200 per thread, the 3 x 168 the launch provides):
//
// * warp 0, TMA producer (lanes 0-15, one box per lane and stage, issued in one instruction): streams the cache
//   through a ring of stages, each `cps` 64-column chunks of 128 tokens, all SWIZZLE_128B. Two layouts:
//     - chunked (64-column-aligned row parts): one 5-D box {64 columns, 8 rows, n chunks, 8-row groups, 1 block} per
//       page (16 rows x 4 chunks = 8 KB at page 16), the 8-row groups landing as consecutive atoms of n KB;
//     - page (any 8-aligned layout): 3-D boxes of `page` rows x 64 columns, 2 chunks per stage.
//   Each lane reads its box's block id once per tile. Pages past the request are all-OOB boxes (zeros). Stage order is
//   software-pipelined across tiles: K(0), K(1) + V(0), K(2) + V(1), ... so that tile i's softmax runs while tile
//   i+1's key chunks are scored and tile i's values stream in. One iteration's key and value chunks are packed into
//   full stages (a stage may end one part and start the next: the host's stage plan, decode_plan_stages), so a row
//   of 16 chunks takes 4 stages of 64 KB whatever its K / V split.
// * warp 1, tcgen05 issuer (one thread; descriptors advance only their low words), M = 128 tokens. The pipe does not
//   queue MMAs, so this thread's instruction stream bounds the tile: it walks host-computed tables (per-stage plan words,
//   per-chunk rebuild runs; DecodeParams::plan / k_rebuild, copied to shared memory at the start) instead of computing
//   chunk ranges, descriptor words and rebuild steps between issues.
//
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
#include <algorithm>

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
constexpr int kRegsWg0 = 104, kRegsWork = 200;   // 104 + 2 * 200 = 3 * 168 registers per SMSP
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
constexpr int bKraw = bQEmpty + 1;            // [2]: the rebuilt keys of a wave of groups are in TMEM
constexpr int bKpeFull = bKraw + 2;
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
// the issuer's tables, copied to shared memory at start: DecodeParams::k_rebuild, then DecodeParams::plan
constexpr int kKinfoBytes = 192;
constexpr int kPlanOff = kKinfoBytes;
constexpr int kTablesBytes = 512;
static_assert(kKinfoBytes >= (kDecodeMaxQChunks - 4) * 16, "k_rebuild");
static_assert(kPlanOff + kDecodeMaxPlan * 16 <= kTablesBytes, "plan");
}  // namespace dec

bool decode_plan_smem(DecodeParams& p) {
  using namespace dec;
  auto up = [](int x, int a) { return (x + a - 1) / a * a; };
  const int q_bytes = up((p.n_k + kG) * kQChunkBytes + 1024, 1024);
  const int b_bytes = p.n_kst * kKstBytes;
  const int fixed = q_bytes + b_bytes + 2 * kPBytes + up(kRedFloats * 4, 128) + kTablesBytes + kNumBars * 8 + 16 + 1024;
  int stages = (kMaxSmem - fixed) / p.stage_bytes;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  p.stages = stages;
  p.off_q = stages * p.stage_bytes;
  p.off_b = p.off_q + q_bytes;
  p.off_p = p.off_b + b_bytes;
  p.off_red = p.off_p + 2 * kPBytes;
  p.off_kinfo = p.off_red + up(kRedFloats * 4, 128);
  p.off_bars = p.off_kinfo + kTablesBytes;
  p.smem_bytes = p.off_bars + kNumBars * 8 + 16 + 1024;
  return p.smem_bytes <= kMaxSmem;
}

bool decode_plan_stages(DecodeParams& p) {
  // Packed: the iteration's n_k key chunks and n_vc value chunks as one run cut every `cps` chunks. The value part
  // starts at position n_k; its O^T blocks are chunk pairs starting at even positions (v_shift = n_k % 2), so a pair
  // never spans two stages (cps is even). Separate (when a shifted value part would need more O^T blocks than TMEM
  // holds): key stages, then value stages.
  const int shift = p.n_k % 2;
  const int n_vp = (p.n_vc + shift + 1) / 2;
  p.packed = n_vp <= kDecodeMaxVPairs ? 1 : 0;
  p.v_shift = p.packed ? shift : 0;
  p.n_vp = (p.n_vc + p.v_shift + 1) / 2;
  p.n_plan = p.packed ? (p.n_k + p.n_vc + p.cps - 1) / p.cps : p.n_ks + p.n_vs;
  if (p.n_plan > kDecodeMaxPlan) return false;
  // Rotation waves. Where the key part spans three or more stages, the groups whose rebuild steps all lie before its
  // last stage form wave 0 and the rotation of their keys starts a stage early (wave 1: the rest, after the key part);
  // the rotation was measured on the critical path there (layers of r_k 576 and 640: 3-5 % faster). Elsewhere all
  // groups form wave 0: one barrier per tile, committed after the key part (starting the rotation earlier there adds
  // TMEM traffic during the key MMAs and measured 1-3 % slower).
  p.kraw_wave = 0;
  const int k_stages = p.packed ? (p.n_k + p.cps - 1) / p.cps : p.n_ks;
  if (k_stages >= 3) {
    const int last_chunk0 = (k_stages - 1) * p.cps;   // first key chunk of the key part's last stage
    bool late = false;
    for (int g = 0; g < kG; ++g) {
      late = late || p.rope_ks1[g] / 4 >= last_chunk0;   // groups in order: once late, the rest are late too
      if (late) p.kraw_wave |= 1 << g;
    }
    if (p.kraw_wave == 0xF) p.kraw_wave = 0;   // no early group: one wave
  }
  // the issuer's words, from the same arithmetic as plan_stage()
  auto atom_of = [&](int nch) { return p.chunked ? nch * p.chunk_stride : p.atom_stride; };
  for (int s = 0; s < p.n_plan; ++s) {
    int k0, kn, v0, vn;
    if (p.packed) {
      const int lo = s * p.cps, hi = std::min(lo + p.cps, p.n_k + p.n_vc);
      k0 = lo;
      kn = std::max(std::min(hi, p.n_k) - lo, 0);
      v0 = std::max(lo - p.n_k, 0);
      vn = std::max(hi - std::max(lo, p.n_k), 0);
    } else if (s < p.n_ks) {
      k0 = p.cps * s;
      kn = std::min(p.cps, p.n_k - k0);
      v0 = vn = 0;
    } else {
      k0 = kn = 0;
      v0 = p.cps * (s - p.n_ks);
      vn = std::min(p.cps, p.n_vc - v0);
    }
    const int j0 = (v0 + p.v_shift) >> 1, j1 = vn ? (v0 + vn + p.v_shift + 1) >> 1 : j0;
    p.plan[s][0] = static_cast<unsigned>(k0 | kn << 8 | v0 << 16 | vn << 24);
    p.plan[s][1] = kn ? desc_hi(static_cast<uint32_t>(atom_of(kn)), kSwizzle128) : 0u;
    p.plan[s][2] = vn ? desc_hi(static_cast<uint32_t>(atom_of(vn)), kSwizzle128) : 0u;
    // wave barriers: wave 0 is committed after the stage holding the last rebuild step of its last group, wave 1 after
    // the key part's last stage
    unsigned waves = 0;
    if (kn) {
      int last0 = -1;
      for (int g = 0; g < kG; ++g)
        if (!((p.kraw_wave >> g) & 1)) last0 = std::max(last0, p.rope_ks1[g] / 4);
      if (last0 >= k0 && last0 < k0 + kn) waves |= 1u;
      if (p.kraw_wave && k0 + kn == p.n_k) waves |= 2u;
    }
    p.plan[s][3] = static_cast<unsigned>(kn * (dec::kTile * 128 >> 4) | j0 << 16 | j1 << 20) | waves << 24;
  }
  return true;
}

// Stage s of an iteration's plan: key chunks [k0, k0 + kn), value chunks [v0, v0 + vn) (an absent part has n = 0).
// Closed-form arithmetic on scalar parameters: the MMA issuer runs it between two stages, and the tensor pipe idles
// while that thread does anything but issue.
struct StagePart {
  int k0, kn, v0, vn;
};

__device__ __forceinline__ StagePart plan_stage(const DecodeParams& p, int s) {
  StagePart r;
  if (p.packed) {
    const int lo = s * p.cps, hi = min(lo + p.cps, p.n_k + p.n_vc);
    r.k0 = lo;
    r.kn = max(min(hi, p.n_k) - lo, 0);
    r.v0 = max(lo - p.n_k, 0);
    r.vn = max(hi - max(lo, p.n_k), 0);
  } else if (s < p.n_ks) {
    r.k0 = p.cps * s;
    r.kn = min(p.cps, p.n_k - r.k0);
    r.v0 = r.vn = 0;
  } else {
    r.k0 = r.kn = 0;
    r.v0 = p.cps * (s - p.n_ks);
    r.vn = min(p.cps, p.n_vc - r.v0);
  }
  return r;
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
  ulonglong2* s_kinfo = reinterpret_cast<ulonglong2*>(smem + p.off_kinfo);   // [n_k]: the two rebuild words
  uint4* s_plan = reinterpret_cast<uint4*>(smem + p.off_kinfo + kPlanOff);     // [n_plan]: the issuer's stage words
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
    mbar_init(&bars[bKraw], 1);
    mbar_init(&bars[bKraw + 1], 1);
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
      int fill_st = 0, fill_rnd = 0;   // fills % S and fills / S, kept incrementally
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
      // One iteration of the plan: the key chunks of a tile (box positions pk; none when !has_k) and the value chunks
      // of the tile before it (pv; none when !has_v). Per stage, lane 0 waits for the slot and arms its barrier with
      // the bytes of both parts, then every lane issues its boxes in the same instruction. The key part lands first
      // in the stage, the value part after the planned key part (kn chunks of the plan x 16 KB on).
      auto load_iteration = [&](bool has_k, const BoxPos& pk, bool has_v, const BoxPos& pv) -> bool {
        for (int s = 0; s < p.n_plan; ++s) {
          const StagePart sp = plan_stage(p, s);
          const int nk = has_k ? sp.kn : 0, nv = has_v ? sp.vn : 0;
          if (nk + nv == 0) continue;
          const int st = fill_st;
          const int rnd = fill_rnd;
          bool got = true;
          if (lane == 0 && rnd > 0)
            got = mbar_wait(&bars[bEmpty + st], (rnd - 1) & 1, abort_flag, p.err, kErrTimeoutProducer);
          if (!__shfl_sync(kLanes, got ? 1 : 0, 0)) return false;
          if (lane == 0) mbar_arrive_expect_tx(&bars[bFull + st], (nk + nv) * kTile * 128);
          __syncwarp(kLanes);
          uint8_t* dst = ring + st * p.stage_bytes;
          uint8_t* dst_v = dst + sp.kn * kTile * 128;   // after the planned key part, present or not
          if constexpr (kChunked) {
            // 5-D box {64 columns, 8 rows, n chunks, box_rows / 8 row groups, 1 block}: every 8-row group lands one
            // atom (n chunks of 1 KB) after the previous one, so a part's atoms are n KB apart
            if (lane < p.n_pieces) {
              if (nk)
                tma_load_5d(dst + lane * (p.box_rows / 8) * nk * p.chunk_stride, &maps.cache[nk - 1],
                            &bars[bFull + st], 0, 0, sp.k0, pk.row / 8, pk.blk);
              if (nv)
                tma_load_5d(dst_v + lane * (p.box_rows / 8) * nv * p.chunk_stride, &maps.cache[nv - 1],
                            &bars[bFull + st], 0, 0, p.v_chunk0 + sp.v0, pv.row / 8, pv.blk);
            }
          } else {
            // 3-D boxes of box_rows rows x 64 columns: box b is piece b % n_pieces of the stage's chunk b / n_pieces
            // (n_pieces divides 16, so every box of a lane has the lane's piece)
            for (int b = lane; b < (nk + nv) * p.n_pieces; b += kProducerLanes) {
              const int h = b / p.n_pieces, pc = b - h * p.n_pieces;
              const bool key = h < nk;
              const BoxPos& bp = key ? pk : pv;
              const int col = key ? 64 * (sp.k0 + h) : p.v_offset + 64 * (sp.v0 + h - nk);
              tma_load_3d(dst + h * p.chunk_stride + pc * p.box_rows * 128, &maps.cache[0], &bars[bFull + st], col,
                          bp.row, bp.blk);
            }
          }
          ++fills;
          if (++fill_st == S) {
            fill_st = 0;
            ++fill_rnd;
          }
        }
        return true;
      };
      TileCursor kc, vc;
      kc.begin(p, seg_begin, seg_end);
      vc.begin(p, seg_begin, seg_end);
      BoxPos pos_k{}, pos_v{};
      // iteration order: K(0); K(1) + V(0); K(2) + V(1); ...; V(last): V(i) reuses the box positions computed for
      // K(i). (Taking V(i) before K(i + 1) where tile i + 1 opens a segment was measured 4 % slower: the MMA issuer
      // then idles while the softmax finishes tile i, with the ring full of value stages.)
      if (kc.valid) {
        pos_k = box_pos(kc);
        ok = load_iteration(true, pos_k, false, pos_v);
        pos_v = pos_k;
        kc.next(p);
      }
      while (ok && vc.valid) {
        const BoxPos cur_v = pos_v;
        const bool has_k = kc.valid;
        if (has_k) pos_k = box_pos(kc);
        if (!(ok = load_iteration(has_k, pos_k, true, cur_v))) break;
        if (has_k) {
          pos_v = pos_k;
          kc.next(p);
        }
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
      int qsegs = 0, vsegs = 0;
      int slot = 0;             // the next stage to consume and the parity of its fill (no division by S)
      uint32_t slot_par = 0;
      bool ok = true;
      auto wait = [&](int bar, uint32_t parity) -> bool {
        return mbar_wait(&bars[bar], parity, abort_flag, p.err, kErrTimeoutMma);
      };
      // No tcgen05 fence after a stage's full barrier: its data was written by TMA (async proxy, completed through the
      // barrier's transaction count), not by threads whose tcgen05 operations need ordering.
      auto full = [&](int& st) -> bool {
        st = slot;
        return wait(bFull + st, slot_par);
      };
      auto release = [&](int st) {   // the stage's MMAs are all issued: its slot is free once they complete
        mma_commit(&bars[bEmpty + st]);
        if (++slot == S) {
          slot = 0;
          slot_par ^= 1u;
        }
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
      // key chunks [c0, c1) of tile i in the stage at a0: per chunk its four score steps into S[i & 1], then the
      // rebuild steps among them (a step holding RoPE coordinates: same A, the group's image as B), read from the
      // chunk's info words, so no per-group loop bookkeeping sits between two MMA issues. (Measured against the
      // previous per-group loop over each stage's steps: config-3 layers 2-5 % faster, c25 rows 10 %; each rebuild
      // issued right after its score step: 1 % slower than after the chunk's scores.)
      // one run of rebuild steps of a chunk at ac (a run word of DecodeParams::k_rebuild; bit 15 clear: none): its MMAs
      // unrolled, one forward branch per further step
      auto mma_rebuild_run = [&](uint32_t w, uint32_t ac, uint32_t hiSw) {
        if (!(w & 0x8000u)) return;
        const uint32_t dK = tmem + kTmemK + 64 * ((w >> 4) & 3u);
        const uint32_t a = ac + 2 * (w & 3u), b = loImg + ((w >> 6) & 63u) * (kKstBytes >> 4);
        const uint32_t acc0 = (w >> 14) & 1u;
        constexpr uint32_t kB = kKstBytes >> 4;
        const uint32_t n = (w >> 2) & 3u;   // the run's length - 1
        mma_ss(dK, desc_of(a, hiSw), desc_of(b, hiImg), idK, acc0);
        if (n >= 1) {
          mma_ss(dK, desc_of(a + 2, hiSw), desc_of(b + kB, hiImg), idK, 1u);
          if (n >= 2) {
            mma_ss(dK, desc_of(a + 4, hiSw), desc_of(b + 2 * kB, hiImg), idK, 1u);
            if (n == 3) mma_ss(dK, desc_of(a + 6, hiSw), desc_of(b + 3 * kB, hiImg), idK, 1u);
          }
        }
      };
      auto mma_key_chunks = [&](int i, uint32_t a0, int c0, int c1, uint32_t hiSw) {
        const uint32_t dS = tmem + 32 * (i & 1);
        uint32_t ac = a0, bq = loQ + c0 * (kQChunkBytes >> 4);
        for (int cc = c0; cc < c1; ++cc, ac += chunk16, bq += kQChunkBytes >> 4) {
          const ulonglong2 rb = s_kinfo[cc];
#pragma unroll
          for (int s16 = 0; s16 < 4; ++s16)
            mma_ss(dS, desc_of(ac + s16 * 2, hiSw), desc_of(bq + s16 * 2, hiQ), idS, (cc | s16) ? 1u : 0u);
          if (rb.y >> 63) {   // the chunk's rebuild steps as at most two runs (host-encoded)
            const uint32_t w0 = static_cast<uint32_t>(rb.y) & 0xFFFFu;
            if ((w0 & 0xCu) == 0xCu) {   // one run of all four steps (the common case): straight-line issue
              const uint32_t dK = tmem + kTmemK + 64 * ((w0 >> 4) & 3u);
              const uint32_t b = loImg + ((w0 >> 6) & 63u) * (kKstBytes >> 4);
#pragma unroll
              for (int s16 = 0; s16 < 4; ++s16)
                mma_ss(dK, desc_of(ac + s16 * 2, hiSw), desc_of(b + s16 * (kKstBytes >> 4), hiImg), idK,
                       s16 ? 1u : (w0 >> 14) & 1u);
            } else {
              mma_rebuild_run(w0, ac, hiSw);
              mma_rebuild_run(static_cast<uint32_t>(rb.y >> 16) & 0xFFFFu, ac, hiSw);
            }
            continue;
          }
#pragma unroll
          for (int s16 = 0; s16 < 4; ++s16) {
            const uint64_t da = desc_of(ac + s16 * 2, hiSw);
            const uint32_t f = static_cast<uint32_t>(rb.x >> (16 * s16)) & 0xFFFFu;
            if (f & 0x8000u)
              mma_ss(tmem + kTmemK + 64 * (f & 3u), da, desc_of(loImg + ((f >> 2) & 63u) * (kKstBytes >> 4), hiImg), idK,
                     (f >> 14) & 1u);
            const uint32_t f2 = static_cast<uint32_t>(rb.y >> (16 * s16)) & 0xFFFFu;
            if (f2 & 0x8000u)
              mma_ss(tmem + kTmemK + 64 * (f2 & 3u), da, desc_of(loImg + ((f2 >> 2) & 63u) * (kKstBytes >> 4), hiImg),
                     idK, (f2 >> 14) & 1u);
          }
        }
      };
      // value chunks [v0, v0 + nv) of tile i in the stage part at av: O^T += V^T P for the O blocks whose chunk pair
      // lies in this part, 128 latent columns (two chunks) at a time
      auto mma_value_chunks = [&](const TileCursor& c, int i, uint32_t av, int v0, uint32_t hiSw, int j0, int j1) {
        const uint32_t p0 = loP + (i & 1) * (kPBytes >> 4);
        const uint32_t first = c.first() ? 1u : 0u;
        const uint32_t pv_step16 = 2 * (hiSw & 0x3FFFu);   // 16 tokens = two atoms (the SBO field, in 16-byte units)
        // the pair's first chunk 2j - v_shift sits at position 2j - v_shift - v0 of the part (-1: the key chunk before
        // the part, whose rows of O^T are never read)
        uint32_t aj = av + (2 * j0 - p.v_shift - v0) * chunk16, dO = tmem + kTmemO + 32 * j0;
        // A = V^T (MN-major SW128, 16 tokens = 2 atoms per step), B = P (MN-major, 16 tokens = 1 KB per step)
        auto block = [&](uint32_t a, uint32_t d) {
#pragma unroll
          for (int s16 = 0; s16 < 8; ++s16)
            mma_ss(d, desc_of(a + s16 * pv_step16, hiSw), desc_of(p0 + s16 * (1024 >> 4), hiP), idV,
                   (first && s16 == 0) ? 0u : 1u);
        };
        if (j1 - j0 == 2) {   // a full stage: both blocks straight-line
          block(aj, dO);
          block(aj + 2 * chunk16, dO + 32);
          return;
        }
        for (int j = j0; j < j1; ++j, aj += 2 * chunk16, dO += 32) block(aj, dO);
      };
      TileCursor kc, vc;
      // One iteration of the plan: the key chunks of tile ik (cursor kc; none when !has_k), then the value chunks of
      // tile iv (cursor vc; none when !has_v), stage by stage as the producer filled them.
      auto mma_iteration = [&](bool has_k, int ik, bool has_v, int iv) -> bool {
        if (has_k) {
          if (kc.first()) {
            if (!wait(bQFull, qsegs & 1)) return false;
            ++qsegs;
          }
          const int sb = ik & 1;
          if (ik >= 2 && !wait(bSFree + sb, ((ik >> 1) - 1) & 1)) return false;
          // The previous tile's RoPE-score MMAs read the rotated keys from the TMEM columns this tile's rebuild
          // overwrites: they were issued before, and tcgen05.mma operations of one thread execute in issue order, so
          // no wait (a wait here would drain the tensor pipe once per tile).
          tc_fence_after();
        }
        bool v_ready = false;
        for (int s = 0; s < p.n_plan; ++s) {
          const uint4 pl = s_plan[s];   // the stage's word (decode_plan_stages)
          const int nk = has_k ? (pl.x >> 8) & 0xFF : 0, nv = has_v ? pl.x >> 24 : 0;
          if (nk + nv == 0) continue;
          int st;
          if (!full(st)) return false;
          const uint32_t a0 = loRing + st * stage16;
          if (nk) {
            const int k0 = pl.x & 0xFF;
            mma_key_chunks(ik, a0, k0, k0 + nk, pl.y);
            // the wave of groups whose last rebuild step is in this stage: its rotation can start once it completes
            if (pl.w & (1u << 24)) mma_commit(&bars[bKraw]);
            if (pl.w & (1u << 25)) mma_commit(&bars[bKraw + 1]);
          }
          if (nv) {
            if (!v_ready) {
              if (!wait(bPFull + (iv & 1), (iv >> 1) & 1)) return false;
              if (vc.first()) {
                if (vsegs > 0 && !wait(bOFree, (vsegs - 1) & 1)) return false;
                ++vsegs;
              }
              tc_fence_after();
              v_ready = true;
            }
            // the value part sits after the planned key part even when this iteration has none, so that chunk -1 of
            // a shifted pair always lies inside the stage
            mma_value_chunks(vc, iv, loRingV + st * stage16 + (pl.w & 0xFFFFu), (pl.x >> 16) & 0xFF, pl.z,
                             (pl.w >> 16) & 0xF, (pl.w >> 20) & 0xF);
          }
          release(st);
        }
        if (has_v) mma_commit(&bars[bPvDone + (iv & 1)]);
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
      kc.begin(p, seg_begin, seg_end);
      vc.begin(p, seg_begin, seg_end);
      ok = wait(bImg, 0);   // the rotation warps' rebuild images
      if (ok && kc.valid) {
        ok = mma_iteration(true, 0, false, 0) && mma_rope(kc, 0);
        kc.next(p);
      }
      for (int v = 0; ok && vc.valid; ++v) {
        const bool more = kc.valid;
        if (!(ok = mma_iteration(more, v + 1, true, v))) break;
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
        if (t < p.n_k) s_kinfo[t] = make_ulonglong2(p.k_rebuild[t][0], p.k_rebuild[t][1]);   // the issuer's rebuilds
        if (t < p.n_plan) s_plan[t] = make_uint4(p.plan[t][0], p.plan[t][1], p.plan[t][2], p.plan[t][3]);
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
        bool got = true;
        int wave = -1;
#pragma unroll 1
        for (int g = 0; g < kG; ++g) {
          // each wave of groups as soon as its rebuild MMAs completed (wave 1 only where the key part spans three or
          // more stages; elsewhere every group is in wave 0, one wait per tile)
          const int wg = (p.kraw_wave >> g) & 1;
          if (wg != wave) {
            wave = wg;
            got = __all_sync(0xffffffffu, mbar_wait(&bars[bKraw + wg], i & 1, abort_flag, p.err, kErrTimeoutEpilogue));
            if (!got) break;
            tc_fence_after();
          }
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
        if (!got) break;
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
            const int f = 128 * j - 64 * p.v_shift + row;   // block j starts at value chunk 2j - v_shift
            if (f >= 0 && f < p.r_v) {
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
