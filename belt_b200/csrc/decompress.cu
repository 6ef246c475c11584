// Keys and values of a range of cached positions, rebuilt from the latent rows on the tensor cores: the prefill
// path's ``LatentLayer.decompress`` (plugins/vllm_lrkv/vllm_lrkv/latent_backend.py:95-108), with the rows gathered
// through the request's block table (latent_backend.py:214-225) inside the kernel:
//     x      = bf16(rows[:, :kc] . rope_up[g]^T)            [S, 64]   gain * B_g c~, rounded as the reference does
//     k_pe   = bf16(NeoX rotation of x at each position)    [S, 64]   (fp32, BF16 cos / sin table)
//     k_nope = bf16(rows[:, :kc] . qmap[g, 64:, :]^T)       [S, 192]
//     v      = bf16(rows[:, v_off : v_off + r_v] . v_up[g]) [S, 256]
//     k[s, g] = [k_pe | k_nope], v[s, g]                    BF16 outputs [count, 4, 256]
//
// Varlen: one launch covers several pieces (a request's positions [pos0, pos0 + count) each, its rows through its own
// block-table row), the outputs of piece i from row piece_out[i]; the CTAs of a piece are consecutive along x.
// One CTA (128 threads) per (two 128-position tiles of a piece, group, part): part 0 the group's keys (N = 256 = 64
// rope + 192 nope rows of wk[g] = [rope_up[g]; qmap[g, 64:]], K = the group's column window, at most five 64-column
// chunks), part 1
// its values (N = 256, K = the value columns). Tiles sit at absolute positions (multiples of 128), so every page box
// covers whole rows of one page; rows outside [pos0, pos0 + count) are computed and dropped. The two tiles of a CTA
// share every weight chunk (two MMAs per K step into two TMEM accumulators): the weights stream once per 256 positions.
//   * thread 0: TMA producer. Per 64-column chunk the tile's rows (one box of min(page, 128) rows x 64 columns per
//     page, K-major, 128-byte swizzle; pages past the request read block num_blocks, i.e. zeros) and the chunk's
//     weights (keys: wk[g] rows x 64 columns, K-major; values: 64 latent rows of v_up[g] x 256, MN-major, with the
//     value part's offset inside the chunk taken up by a negative row coordinate, zero-filled) into a 3-stage ring;
//   * thread 32: tcgen05 issuer, M = 128 positions per tile, N = 256, four K = 16 instructions per chunk and tile, D
//     in TMEM (tile t at columns 256 t);
//   * all four warps: epilogue, one position of each tile per thread: BF16 rounding, the RoPE rotation of the key's
//     first 64 channels, 16-byte stores.
#include "common.cuh"
#include "launch.h"

namespace belt {

namespace {
constexpr int kDcThreads = 128;
constexpr int kDcABytes = 128 * 128;              // 128 rows x 64 columns
constexpr int kDcBBytes = 256 * 128;              // 256 weight rows x 64 columns (or 64 x 256)
constexpr int kDcTiles = 2;                       // 128-position tiles per CTA
constexpr int kDcStage = kDcTiles * kDcABytes + kDcBBytes;   // 64 KB
constexpr int kDcStages = 3;
constexpr int kDcBars = 2 * kDcStages + 1;        // full[S], empty[S], done
}  // namespace

__global__ void __launch_bounds__(kDcThreads, 1)
    decompress_kernel(const __grid_constant__ DecompressMaps maps, const __grid_constant__ DecompressParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDcStages * kDcStage);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kDcBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  int pi = 0;   // this CTA's piece
  while (pi + 1 < p.num_pieces && static_cast<int>(blockIdx.x) >= p.piece_cta0[pi + 1]) ++pi;
  const int seq_len = p.piece_len[pi], pos0 = p.piece_pos0[pi], count = p.piece_count[pi];
  const int32_t* block_table = p.block_table + static_cast<long long>(p.piece_req[pi]) * p.bt_stride;
  const long long out_row0 = p.piece_out[pi];
  const int tile_pos = (pos0 / 128 + kDcTiles * (static_cast<int>(blockIdx.x) - p.piece_cta0[pi])) * 128;
  const int g = blockIdx.y;
  const bool values = blockIdx.z != 0;
  const int nchunks = values ? p.v_nch : p.k_nch[g];
  const int box_rows = p.page < 128 ? p.page : 128;
  const int n_boxes = 128 / box_rows;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kDcBars; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.cache);
    tma_prefetch_desc(values ? &maps.v : &maps.wk);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 256 * kDcTiles);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    // ---------------------------------------------------------------- producer
    // the tile's page boxes: block id and first row of every box (positions past the request read as zeros)
    int blk[kDcTiles][8], row0[kDcTiles][8];
    const int npages = (seq_len + p.page - 1) / p.page;
    for (int t = 0; t < kDcTiles; ++t)
      for (int b = 0; b < n_boxes; ++b) {
        const int pos = tile_pos + 128 * t + b * box_rows;
        const int pg = pos / p.page;
        blk[t][b] = pg < npages ? __ldg(block_table + pg) : p.num_blocks;
        row0[t][b] = pos - pg * p.page;
      }
    int issued = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % kDcStages;
      if (c >= kDcStages &&
          !mbar_wait(&bars[kDcStages + s], ((c / kDcStages) - 1) & 1, abort_flag, p.err, kErrTimeoutProducer)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* st = smem + s * kDcStage;
      const int chunk = values ? p.v_chunk0 + c : p.k_chunk[g][c];
      mbar_arrive_expect_tx(&bars[s], kDcStage);
      for (int t = 0; t < kDcTiles; ++t)
        for (int b = 0; b < n_boxes; ++b)
          tma_load_3d(st + t * kDcABytes + b * box_rows * 128, &maps.cache, &bars[s], 64 * chunk, row0[t][b],
                      blk[t][b]);
      if (values) {
        // latent rows v = 64 * chunk - v_offset .. + 64 of v_up[g] (negative or past r_v: zeros), 4 x 64 columns
        const int vrow = 64 * chunk - p.v_offset;
#pragma unroll
        for (int nb = 0; nb < 4; ++nb)
          tma_load_3d(st + kDcTiles * kDcABytes + nb * (64 * 128), &maps.v, &bars[s], 64 * nb, vrow, g);
      } else {
        tma_load_3d(st + kDcTiles * kDcABytes, &maps.wk, &bars[s], 64 * chunk, 0, g);
      }
      ++issued;
    }
    if (*abort_flag)   // let the copies already issued land before the CTA's shared memory goes away
      for (int c = issued > kDcStages ? issued - kDcStages : 0; c < issued; ++c)
        mbar_wait_bounded(&bars[c % kDcStages], (c / kDcStages) & 1, nullptr, 0, kWaitCycles / 8);
  } else if (threadIdx.x == 32) {
    // ---------------------------------------------------------------- tcgen05 issuer
    constexpr uint32_t idK = idesc_bf16(128, 256, 0, 0);   // A K-major, B K-major (wk rows)
    constexpr uint32_t idV = idesc_bf16(128, 256, 0, 1);   // A K-major, B MN-major (v_up)
    constexpr uint32_t hiSw = desc_hi(1024, kSwizzle128);
    const uint32_t base = smem_u32(smem);
    bool ok = true;
    for (int c = 0; c < nchunks && ok; ++c) {
      const int s = c % kDcStages;
      if (!(ok = mbar_wait(&bars[s], (c / kDcStages) & 1, abort_flag, p.err, kErrTimeoutMma))) break;
      tc_fence_after();
      const uint32_t st = base + s * kDcStage;
      const uint32_t sb = st + kDcTiles * kDcABytes;
      uint64_t da = desc_of(desc_lo(st, 16), hiSw);
      // keys: 256 K-major rows of 128 bytes (SBO 1 KB); values: MN-major, LBO = the next 64-column block (8 KB)
      uint64_t db = values ? desc_of(desc_lo(sb, 64 * 128), hiSw) : desc_of(desc_lo(sb, 16), hiSw);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int t = 0; t < kDcTiles; ++t)
          mma_ss(tmem + 256 * t, da + t * (kDcABytes >> 4), db, values ? idV : idK, (c | kk) != 0 ? 1u : 0u);
        da += 2;                              // 16 columns = 32 bytes along the swizzled row
        db += values ? (2048 >> 4) : 2;       // values: 16 latent rows = 2 KB; keys: 32 bytes along the row
      }
      mma_commit(&bars[kDcStages + s]);
    }
    if (!ok) *abort_flag = 1;
    mma_commit(&bars[2 * kDcStages]);   // arrives once the MMAs issued are done
  }
  __syncwarp();

  // -------------------------------------------------------------------- epilogue
  const bool done = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[2 * kDcStages], 0, p.err, kErrTimeoutEpilogue));
  tc_fence_after();
  for (int t = 0; t < kDcTiles; ++t) {
    if (done && !*abort_flag && nchunks == 0) {   // a group without columns: zero keys / values
      const int pos = tile_pos + 128 * t + threadIdx.x;
      if (pos >= pos0 && pos < pos0 + count) {
        uint4* dst = reinterpret_cast<uint4*>((values ? p.v_out : p.k_out) + (out_row0 + pos - pos0) * p.out_st +
                                              static_cast<long long>(g) * p.out_sg);
        for (int q = 0; q < 32; ++q) dst[q] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    if (done && !*abort_flag && nchunks > 0) {
      const int pos = tile_pos + 128 * t + threadIdx.x;
      const bool keep = pos >= pos0 && pos < pos0 + count;
      __nv_bfloat16* out = (values ? p.v_out : p.k_out) + (out_row0 + pos - pos0) * p.out_st +
                           static_cast<long long>(g) * p.out_sg;
      const uint32_t taddr = tmem + 256 * t + (static_cast<uint32_t>(warp * 32) << 16);
      int c0 = 0;
      if (!values) {
        // RoPE channels: x = bf16(acc), NeoX rotation in fp32 at the position, BF16
        uint32_t x[32], y[32];
        tmem_ld32(taddr, x);
        tmem_ld32(taddr + 32, y);
        tmem_ld_wait();
        if (keep) {
          const __nv_bfloat16* cs = p.cos_sin + static_cast<long long>(pos < p.max_pos ? pos : p.max_pos - 1) * 64;
          uint32_t o1[16], o2[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float r1[2], r2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int i = 2 * j + e;
              const float x1 = bf16_round(__uint_as_float(x[i])), x2 = bf16_round(__uint_as_float(y[i]));
              const float cv = __bfloat162float(cs[i]), sv = __bfloat162float(cs[32 + i]);
              r1[e] = x1 * cv - x2 * sv;
              r2[e] = x2 * cv + x1 * sv;
            }
            o1[j] = pack_bf16(r1[0], r1[1]);
            o2[j] = pack_bf16(r2[0], r2[1]);
          }
          uint4* d1 = reinterpret_cast<uint4*>(out);
          uint4* d2 = reinterpret_cast<uint4*>(out + 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            d1[q] = make_uint4(o1[4 * q], o1[4 * q + 1], o1[4 * q + 2], o1[4 * q + 3]);
            d2[q] = make_uint4(o2[4 * q], o2[4 * q + 1], o2[4 * q + 2], o2[4 * q + 3]);
          }
        }
        c0 = 64;
      }
#pragma unroll 1
      for (; c0 < 256; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c0, r);
        tmem_ld_wait();
        if (!keep) continue;
        uint4* dst = reinterpret_cast<uint4*>(out + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf16(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1])),
                              pack_bf16(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                              pack_bf16(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                              pack_bf16(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256 * kDcTiles);
  }
}

int decompress_smem_bytes() { return 1024 + kDcStages * kDcStage + kDcBars * 8 + 16; }

// CTAs (along x) of a piece of `count` positions from pos0: pairs of 128-position tiles at absolute multiples of 128.
int decompress_piece_ctas(int pos0, int count) {
  if (count <= 0) return 0;
  const int first = pos0 / 128, last = (pos0 + count - 1) / 128;
  return (last - first + kDcTiles) / kDcTiles;
}

cudaError_t launch_decompress(const DecompressMaps& maps, const DecompressParams& p, cudaStream_t stream) {
  const int total = p.piece_cta0[p.num_pieces];
  if (total == 0) return cudaSuccess;
  const int smem = decompress_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(decompress_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(total, kG, 2);
  decompress_kernel<<<grid, kDcThreads, smem, stream>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace belt
