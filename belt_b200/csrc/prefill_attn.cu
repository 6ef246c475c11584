// Prefill attention on the tensor cores: the new tokens of one request attend over keys and values rebuilt from its
// cache rows (belt_latent_decompress), the operation the reference hands to flash_attn_varlen_func
// (plugins/vllm_lrkv/vllm_lrkv/latent_backend.py:285-320): softmax(scale q k^T) v per query head, heads sharing
// their group's keys (24 query heads, 4 groups, head dim 256), causal by position, with the natural-log LSE of every
// (query, head) so that the backend can fold context chunks together.
//
// Varlen: one launch covers several pieces, each the queries of one request over a range of its keys (rows of the
// concatenated query and key / value buffers, at their own positions), its output and LSE rows in `out` / `lse` or in
// `out2` / `lse2`; the query tiles of a piece are consecutive along grid x.
// One CTA per (128-query tile of a piece, head), 224 threads:
//   * warp 0, lane 0: TMA producer of the query tile (128 x 256, K-major, 4 chunks of 64 columns, 128-byte swizzle)
//     once and of the key tiles (same layout), warp 6, lane 0: producer of the value tiles (read as the MN-major B
//     operand: 128 key rows of 64 channels per chunk). Each buffer holds one tile; the key buffer is refilled chunk
//     by chunk as the score MMAs release its chunks, the value buffer as a whole once P.V has read it;
//   * warp 1, lane 0: tcgen05 issuer. S = Q K^T (M = 128 queries, N = 128 keys, 16 steps of K = 16) into TMEM,
//     then O += P V with P read from TMEM (M = 128, N = 256, 8 steps), software-pipelined: S of tile j + 1 is
//     computed while the softmax turns S of tile j into P;
//   * warps 2-5: softmax, one query row per thread (its TMEM lane): scale, mask (keys past the end or, causally,
//     after the query's position), running max in the exp2 domain (O rescaled in TMEM only when a row's max grows by
//     more than 2^8), P = exp2(s - m) packed to BF16 into TMEM, row sums in fp32; at the end O / l to BF16 and the
//     LSE.
// TMEM: S [0, 128), P [128, 192) (BF16 pairs), O [256, 512).
// Every wait is bounded: a timeout records an error code and the CTA drains its copies and exits.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
// 2^x with the SFU's approximation (ex2.approx, flush to zero; 2^-inf = 0): P is rounded to BF16 afterwards
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr int kPaThreads = 224;
constexpr int kPaTile = 128;
constexpr int kPaChunk = 128 * 128;             // 128 rows x 64 channels (BF16), one swizzled chunk
constexpr int kPaTileBytes = 4 * kPaChunk;      // 128 x 256 = 64 KB
constexpr int kPaQ = 0, kPaK = kPaTileBytes, kPaV = 2 * kPaTileBytes;
constexpr int kPaSmem = 3 * kPaTileBytes;       // + barriers
constexpr uint32_t kTmS = 0, kTmP = 128, kTmO = 256;
// barriers: the key and value buffers are released and refilled per 64-channel chunk
constexpr int aQ = 0, aKFull = 1, aKEmpty = 5, aVFull = 9, aVEmpty = 13, aSFull = 17, aSFree = 18, aPFull = 19,
              aPvDone = 20, aDrain = 21, kPaBars = 22;
}  // namespace

__global__ void __launch_bounds__(kPaThreads, 1)
    prefill_attn_kernel(const __grid_constant__ PrefillAttnMaps maps, const __grid_constant__ PrefillAttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPaSmem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kPaBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int pi = 0;   // this CTA's piece
  while (pi + 1 < p.num_pieces && static_cast<int>(blockIdx.x) >= p.piece_cta0[pi + 1]) ++pi;
  const int ql = p.piece_ql[pi], S = p.piece_S[pi], q_pos0 = p.piece_q_pos0[pi], k_pos0 = p.piece_k_pos0[pi];
  const int q_row = p.piece_q_row[pi], k_row = p.piece_k_row[pi];
  const int i0 = (static_cast<int>(blockIdx.x) - p.piece_cta0[pi]) * kPaTile, h = blockIdx.y, g = h / p.hpg;
  const int q_last = min(i0 + kPaTile, ql) - 1;   // last live query of the tile
  // key tiles to visit: all of them, or causally those holding a key at or before the tile's last query position
  int n_tiles = (S + kPaTile - 1) / kPaTile;
  if (p.causal) {
    const long long last_key = static_cast<long long>(q_pos0) + q_last - k_pos0;   // last key index allowed
    const long long lim = last_key < 0 ? 0 : last_key / kPaTile + 1;
    n_tiles = static_cast<int>(lim < n_tiles ? lim : n_tiles);
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPaBars; ++i) mbar_init(&bars[i], (i == aSFree || i == aPFull) ? 4 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.q);
    tma_prefetch_desc(&maps.k);
    tma_prefetch_desc(&maps.v);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // one chunk ring per buffer (keys: warp 0, values: warp 6): chunk c of tile j waits until the MMAs of tile j - 1
  // that read chunk c completed, so the next tile streams in while the current one is still being multiplied
  // nchunk = 4: one barrier pair per 64-channel chunk; nchunk = 1: the whole tile under the first pair
  auto stream_chunks = [&](const CUtensorMap* map, int off, int full0, int empty0, int nchunk, int err_code) {
    int issued[4] = {0, 0, 0, 0};
    bool ok = true;
    const int per = 4 / nchunk;
    for (int j = 0; ok && j < n_tiles; ++j)
#pragma unroll 1
      for (int c = 0; c < nchunk; ++c) {
        if (j > 0 && !(ok = mbar_wait(&bars[empty0 + c], (j - 1) & 1, abort_flag, p.err, err_code))) break;
        mbar_arrive_expect_tx(&bars[full0 + c], per * kPaChunk);
        for (int q = 0; q < per; ++q)
          tma_load_3d(smem + off + (c * per + q) * kPaChunk, map, &bars[full0 + c], 64 * (c * per + q), g,
                      k_row + j * kPaTile);
        ++issued[c];
      }
    if (*abort_flag)   // the latest copy into every chunk lands before the CTA's shared memory goes away
      for (int c = 0; c < nchunk; ++c)
        if (issued[c]) mbar_wait_bounded(&bars[full0 + c], (issued[c] - 1) & 1, nullptr, 0, kWaitCycles / 8);
  };
  if (warp == 0) {
    // ---------------------------------------------------------------- key producer (and the query tile)
    if (lane == 0 && n_tiles > 0) {
      mbar_arrive_expect_tx(&bars[aQ], kPaTileBytes);
#pragma unroll
      for (int c = 0; c < 4; ++c) tma_load_3d(smem + kPaQ + c * kPaChunk, &maps.q, &bars[aQ], 64 * c, h, q_row + i0);
      stream_chunks(&maps.k, kPaK, aKFull, aKEmpty, 4, kErrTimeoutProducer);
      if (*abort_flag) mbar_wait_bounded(&bars[aQ], 0, nullptr, 0, kWaitCycles / 8);
    }
    __syncwarp();
  } else if (warp == 6) {
    // ---------------------------------------------------------------- value producer
    if (lane == 0 && n_tiles > 0) stream_chunks(&maps.v, kPaV, aVFull, aVEmpty, 1, kErrTimeoutProducer);
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- tcgen05 issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);   // Q K-major, K K-major
      constexpr uint32_t idO = idesc_bf16(128, 256, 0, 1);   // P from TMEM, V MN-major (four 64-channel blocks)
      constexpr uint32_t hiSw = desc_hi(1024, kSwizzle128);
      const uint32_t base = smem_u32(smem);
      bool ok = true;
      auto wait = [&](int bar, uint32_t parity) -> bool {
        return mbar_wait(&bars[bar], parity, abort_flag, p.err, kErrTimeoutMma);
      };
      auto qk = [&](int j) -> bool {
        if (j > 0 && !wait(aSFree, (j - 1) & 1)) return false;   // the softmax has read S of the previous tile
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          if (!wait(aKFull + c, j & 1)) return false;
          tc_fence_after();
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint32_t off = c * kPaChunk + s * 32;
            mma_ss(tmem + kTmS, desc_of(desc_lo(base + kPaQ + off, 16), hiSw),
                   desc_of(desc_lo(base + kPaK + off, 16), hiSw), idS, (c | s) ? 1u : 0u);
          }
          mma_commit(&bars[aKEmpty + c]);   // key chunk c of this tile read
        }
        mma_commit(&bars[aSFull]);
        return true;
      };
      auto pv = [&](int j) -> bool {
        if (!wait(aPFull, j & 1)) return false;
        if (!wait(aVFull, j & 1)) return false;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          // A = P (TMEM, 16 keys = 8 columns per step), B = V: 16 key rows = 2 KB per step, 64-channel blocks 16 KB
          mma_ts(tmem + kTmO, tmem + kTmP + 8 * s, desc_of(desc_lo(base + kPaV + s * 2048, kPaChunk), hiSw), idO,
                 (j | s) ? 1u : 0u);
        mma_commit(&bars[aVEmpty]);
        mma_commit(&bars[aPvDone]);
        return true;
      };
      ok = wait(aQ, 0) && qk(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles && !(ok = qk(j + 1))) break;
        if (!(ok = pv(j))) break;
      }
      if (*abort_flag) {   // the MMAs issued complete before TMEM is freed
        mma_commit(&bars[aDrain]);
        mbar_wait_bounded(&bars[aDrain], 0, nullptr, 0, kWaitCycles / 8);
      }
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---------------------------------------------------------------- softmax warps (rows of TMEM lane quadrant)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int qi = i0 + row;
    const bool live_row = qi < ql;
    const long long qpos = static_cast<long long>(q_pos0) + qi;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    auto ewait = [&](int bar, uint32_t parity) -> bool {
      const bool r = mbar_wait(&bars[bar], parity, abort_flag, p.err, kErrTimeoutEpilogue);
      return __all_sync(0xffffffffu, r);
    };
    for (int j = 0; j < n_tiles; ++j) {
      if (!(ok = ewait(aSFull, j & 1))) break;
      tc_fence_after();
      float s[128];
      {
        uint32_t r[4][32];   // the four loads in flight together, one wait
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + kTmS + 32 * c, r[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) s[32 * c + e] = __uint_as_float(r[c][e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[aSFree]);
      // keys of this tile the row sees: all (no mask work), none, or a prefix (causal diagonal, the last tile)
      const int k0 = j * kPaTile;
      long long kv = S - k0;
      if (p.causal) {
        const long long lim = qpos - k_pos0 - k0 + 1;
        kv = lim < kv ? lim : kv;
      }
      const int nvis = !live_row ? 0 : kv <= 0 ? 0 : kv >= kPaTile ? kPaTile : static_cast<int>(kv);
      float mx = -INFINITY;
      if (nvis == kPaTile) {
#pragma unroll
        for (int e = 0; e < 128; ++e) mx = fmaxf(mx, s[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 128; ++e) {
          s[e] = e < nvis ? s[e] : -INFINITY;
          mx = fmaxf(mx, s[e]);
        }
      }
      mx *= p.scale_log2;   // the row's tile max in the exp2 domain (-inf when it sees no key)
      // the previous tile's P.V has read P and written O: P can be overwritten, O rescaled
      if (j > 0 && !(ok = ewait(aPvDone, (j - 1) & 1))) break;
      tc_fence_after();
      // lazy rescale: a row's running max is raised only when the tile's max exceeds it by more than 2^8; the O
      // rescale (TMEM loads and stores, warp-collective) runs when any row of the warp needs it, alpha 1 elsewhere
      float alpha = 1.f;
      if (mx > m_run + 8.f) {
        alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - mx);
        m_run = mx;
        l_run *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kTmO + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tmem + lane_base + kTmO + 32 * c, o);
        }
        tmem_st_wait();
      }
      // P = exp2(scale s - m): one FFMA and one EX2 per key (masked keys hold -inf and give 0; a row that has seen no
      // key yet uses m = 0, its scores are all -inf)
      const float mu = m_run == -INFINITY ? 0.f : m_run;
      uint32_t pk0[32], pk1[32];
      float sum = 0.f;
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const float a = fast_exp2(fmaf(s[2 * e], p.scale_log2, -mu));
        const float b = fast_exp2(fmaf(s[2 * e + 1], p.scale_log2, -mu));
        sum += a + b;
        if (e < 32) pk0[e] = pack_bf16(a, b);
        else pk1[e - 32] = pack_bf16(a, b);
      }
      l_run += sum;
      tmem_st32(tmem + lane_base + kTmP, pk0);
      tmem_st32(tmem + lane_base + kTmP + 32, pk1);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[aPFull]);
    }
    // ---------------------------------------------------------------- epilogue: O / l, LSE
    if (ok && n_tiles > 0) ok = ewait(aPvDone, (n_tiles - 1) & 1);
    tc_fence_after();
    if (ok && !*abort_flag) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const bool to2 = p.piece_to2[pi] != 0;
      const long long orow = static_cast<long long>(p.piece_o_row[pi]) + qi;
      __nv_bfloat16* out = (to2 ? p.out2 : p.out) + orow * p.out_st + static_cast<long long>(h) * p.out_sh;
      float* lse_out = to2 ? p.lse2 : p.lse;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t o[32];
        if (n_tiles > 0) {
          tmem_ld32(tmem + lane_base + kTmO + 32 * c, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (!live_row) continue;
        uint4* dst = reinterpret_cast<uint4*>(out + 32 * c);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf16(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                              pack_bf16(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                              pack_bf16(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                              pack_bf16(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
      }
      if (live_row && lse_out)
        lse_out[orow * p.lse_st + h] =
            l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994530942f : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int prefill_attn_smem_bytes() { return 1024 + kPaSmem + kPaBars * 8 + 16; }

cudaError_t launch_prefill_attn(const PrefillAttnMaps& maps, const PrefillAttnParams& p, cudaStream_t stream) {
  const int total = p.piece_cta0[p.num_pieces];
  if (total == 0) return cudaSuccess;
  const int smem = prefill_attn_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(total, p.H);
  prefill_attn_kernel<<<grid, kPaThreads, smem, stream>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace belt
