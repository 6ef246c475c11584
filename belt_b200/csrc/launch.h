// Kernel parameter blocks and launchers shared by the kernels and the C-ABI layer (capi.cu).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace belt {

constexpr int kDecodeMaxKsteps = 20;   // rebuild K-steps: <= 5 per group (64 coordinates at any 16-column offset)
constexpr int kDecodeMaxVPairs = 5;    // O^T blocks of 128 latent columns: r_v <= 640
constexpr int kDecodeMaxQChunks = 16;  // n_k + 4 query chunks of 64 columns: v_offset <= 768
constexpr int kDecodeMaxPlan = 12;     // stages of one ring iteration: ceil((12 + 10) / 2) at 2 chunks a stage

struct DecodeParams {
  const int32_t* block_table;
  long long bt_stride;
  const int32_t* seq_lens;
  const int32_t* work;
  const int32_t* cta_seg;
  const __nv_bfloat16* rope_blocks;   // [64, rope_ld]
  int rope_ld;
  const __nv_bfloat16* cos_sin;       // [max_pos, 64]
  int max_pos;
  float* part;
  long long part_ss, part_sh;
  int* err;
  unsigned long long* cta_ns;         // may be null: per CTA, += ns from the predecessor's completion to the CTA's exit
  int num_reqs;
  int num_blocks, page;
  // cache stages: a stage holds `cps` 64-column chunks of 128 tokens. Chunked layout (4-D boxes of 8 rows x nch
  // chunks): chunks 1 KB apart, 8-token atoms 4 KB apart. Page layout (3-D boxes of box_rows rows x 64 columns): chunks
  // 16 KB apart, atoms 1 KB apart.
  int chunked, cps, chunk_stride, atom_stride, stage_bytes;
  int box_rows, n_pieces;             // page layout: rows per box, boxes per chunk of a tile
  int n_k, n_ks;                      // key-part chunks and stages
  int v_offset, v_chunk0, r_v, n_vc, n_vs, n_vp;   // value part: first column (chunk), rank, chunks, stages, O blocks
  // Stage plan of one iteration of the ring: the key chunks of tile i + 1, then the value chunks of tile i, in n_plan
  // stages of at most `cps` chunks (plan_stage() in decode.cu). Packed: the n_k + n_vc chunks cut every cps chunks,
  // so one stage can carry the end of the key part and the start of the value part; otherwise n_ks key stages, then
  // n_vs value stages. O^T block j covers value chunks 2j - v_shift and 2j + 1 - v_shift (v_shift = 1 when the value
  // part starts at an odd position of a packed plan, so that no block spans two stages; chunk -1 is a key chunk and
  // feeds rows that are never read).
  int packed, n_plan, v_shift;
  // the plan's stages for the MMA issuer, one 16-byte word each (decode_plan_stages): x = k0 | kn << 8 | v0 << 16 |
  // vn << 24; y, z = the high descriptor words of the key and value parts' SWIZZLE_128B atoms; w = the value part's
  // offset in the stage (16-byte units) | first O^T block << 16 | end block << 20 | commit the rotation-wave barriers
  // after this stage's key chunks << 24 (bit 0: wave 0, bit 1: wave 1)
  unsigned int plan[kDecodeMaxPlan][4];
  int kraw_wave;                      // bit g: group g's keys are rotated in wave 1 (decode_plan_stages)
  int n_kst;
  int kst_src[kDecodeMaxKsteps];      // rebuild image e: rope_blocks columns [kst_src[e], kst_src[e] + 16)
  // per group: first and last 16-column step holding its RoPE coordinates, and the image of the first step (the
  // steps of a group are consecutive images)
  int rope_ks0[4], rope_ks1[4], rope_e0[4];
  // per key chunk, the rebuild MMAs of its four 16-column steps (16 bits each, step s at bit 16 s): bit 15 a rebuild
  // step, bit 14 accumulate (not the group's first step), bits 2-7 its image, bits 0-1 its group. Word 1 holds a
  // second group's rebuild where one step holds the end of one group's RoPE coordinates and the start of the next
  // (8-column aligned runs: at most two per step), or, with bit 63 set, the chunk's rebuild steps as at most two runs
  // of consecutive steps (run r in bits 16 r .. 16 r + 15: bit 15 | step 0's accumulate flag << 14 | first image << 6
  // | group << 4 | (count - 1) << 2 | first step), which the issuer emits without per-step tests.
  unsigned long long k_rebuild[kDecodeMaxQChunks - 4][2];
  float scale_log2;
  // shared-memory layout (byte offsets from the 1024-aligned base), set by the host launcher
  int stages;
  int off_q, off_b, off_p, off_red, off_kinfo, off_bars, smem_bytes;
};

// Tensor maps of one decode launch: the cache (page layout: cache[0] only; chunked layout: cache[n - 1] fetches n
// chunks) and the block-diagonal query.
struct DecodeMaps {
  CUtensorMap cache[4];
  CUtensorMap q;
};

cudaError_t launch_latent_decode(const DecodeMaps& maps, const DecodeParams& p, int num_ctas, cudaStream_t stream);
// Fills p.stages and the shared-memory offsets; returns false if the layout does not fit.
bool decode_plan_smem(DecodeParams& p);
// Chooses the stage plan (packed, n_plan, v_shift, n_vp, plan) from n_k, n_vc, cps, n_ks, n_vs and the layout;
// false if it has more stages than kDecodeMaxPlan.
bool decode_plan_stages(DecodeParams& p);

// Out[t, g * hpg + j, n] = X[t, g * hpg + j, :] @ W[g, :, n] for n in the group's column runs, 0 elsewhere.
struct GroupGemmParams {
  const __nv_bfloat16* X;
  long long sxt, sxh;
  const __nv_bfloat16* W;
  long long swg, swk, swn;
  __nv_bfloat16* Out;
  long long sot, soh;
  int T, K, N, hpg, G;
  int nruns[4];
  int run_lo[4][3], run_hi[4][3];
};
cudaError_t launch_group_gemm(const GroupGemmParams& p, cudaStream_t stream);

// The same product on the tensor cores (head_gemm.cu): X and W through TMA maps, Out written directly.
//   maps.x: 3-D {K, heads, T} over X (strides sxh, sxt), box {64, 1, 128};
//   maps.w: 3-D {N, K, G} over W (strides swk, swg; swn = 1), box {64, 64, 1}.
struct HeadGemmMaps {
  CUtensorMap x;
  CUtensorMap w;
};
struct HeadGemmParams {
  __nv_bfloat16* Out;
  long long sot, soh;
  int T, K, N, hpg, G;
  int nruns[4];
  int run_lo[4][3], run_hi[4][3];
  int nb;        // column tile = 64 * nb (1, 2 or 4)
  int vec_out;   // Out rows 16-byte aligned: 16-byte stores
  int stages;    // set by the launcher
  int* err;
};
cudaError_t launch_head_gemm(const HeadGemmMaps& maps, HeadGemmParams p, cudaStream_t stream);

struct ScheduleParams {
  const int32_t* seq_lens;
  int num_reqs, num_ctas, min_tiles, tile;
  int unit, start_cost;   // cost of a tile and extra cost of a request's first tile (1, 0: the reference's split)
  int32_t* work;
  long long work_capacity;
  int32_t* cta_seg;
  int32_t* seg_base;
  int* err;
  // balanced split (all three or none): per CTA the decode time of the previous step (read, then zeroed), its speed
  // weight (updated in place) and the cost it was dealt (written)
  long long* cta_ns;
  float* cta_w;
  long long* cta_cap;
};
cudaError_t launch_schedule(const ScheduleParams& p, cudaStream_t stream);

struct MergeParams {
  const float* part;
  long long ps, ph;
  const int32_t* seg_base;
  int num_reqs, nh, lv;
  __nv_bfloat16* out;
  long long sob, soh;
  float* lse;
  long long slb;
};
cudaError_t launch_merge(const MergeParams& p, cudaStream_t stream);

// Segment merge + V up-projection (merge_up.cu): maps.v 3-D {256, r_v, G} over U_v^T [G, r_v, 256], box {64, 64, 1}.
struct MergeUpMaps {
  CUtensorMap v;
};
struct MergeUpParams {
  const float* part;
  long long ps, ph;
  const int32_t* seg_base;
  int num_reqs, nh, hpg, lv;
  __nv_bfloat16* out;
  long long sot, soh;
  float* lse;          // may be null
  long long slb;
  int* err;
  int vec_part;        // part rows 16-byte aligned and lv % 4 == 0: float4 loads of the partial rows
  int vec_out;         // out 16-byte aligned, strides multiples of 8: 16-byte stores
};
cudaError_t launch_merge_up(const MergeUpMaps& maps, const MergeUpParams& p, cudaStream_t stream);

struct CacheWriteParams {
  const __nv_bfloat16* c;
  long long sct;
  const void* slots;
  int slots_i64;
  __nv_bfloat16* cache;
  long long sblk, stok;
  int page, W, lk, T, G;
  long long num_slots;
  const __nv_bfloat16* u_cat;   // [lk, G * 256]
  int a_lo[4], a_n[4], b_lo[4], b_n[4];
  float eps;
};
cudaError_t launch_cache_write(const CacheWriteParams& p, cudaStream_t stream);

// Fused latent cache write (proj_write.cu): c = bf16(x W_down^T), the RMS fold of every K group, paged scatter.
//   maps.x: 2-D {hidden, T} over x, box {64, 128}; maps.w: 2-D {hidden, W} over W_down, box {64, 64};
//   maps.u: 2-D {G * 256, lk} over u_cat, box {64, 64}.
// Work items: KV groups 0..G-1, then chunks of the V part [lk, W); item i covers the 64-column chunks
// item_chunk[i][0 .. item_nch[i]) of the row (ascending).
constexpr int kPwMaxChunks = 5;
constexpr int kPwMaxItems = 16;
struct ProjWriteMaps {
  CUtensorMap x;
  CUtensorMap w;
  CUtensorMap u;
};
struct ProjWriteParams {
  const void* slots;
  int slots_i64;
  long long num_slots;
  __nv_bfloat16* cache;
  long long sblk, stok;
  int page, W, lk, T, hidden, G;
  int a_lo[4], a_n[4], b_lo[4], b_n[4];
  int n_items;
  int item_nch[kPwMaxItems];
  int item_chunk[kPwMaxItems][kPwMaxChunks];
  float eps;
  int vec_ok;   // cache rows 16-byte aligned
  int* err;
  // c-input mode (latent_rows_to_cache): the latent rows come from c [T, >= W] (row stride sct elements) instead of
  // x W_down^T; maps.x / maps.w are then unused. c_vec: c rows 16-byte aligned.
  const __nv_bfloat16* c;
  long long sct;
  int c_in, c_vec;
};
cudaError_t launch_proj_write(const ProjWriteMaps& maps, const ProjWriteParams& p, cudaStream_t stream);

// Keys and values of cached positions rebuilt from the latent rows (decompress.cu).
struct DecompressMaps {
  CUtensorMap cache;   // {W, page, blocks}, box {64, min(page, 128), 1}
  CUtensorMap wk;      // [4, 256, kc] key weights, box {64, 256, 1}
  CUtensorMap v;       // v_up [4, r_v, 256], box {64, 64, 1}
};
// Varlen launches (decompress, prefill attention, fold) carry a table of up to kVarlenMax pieces in their parameters;
// the C ABI splits longer lists into several launches.
constexpr int kVarlenMax = 64;
struct DecompressParams {
  const int32_t* block_table;   // [requests, >= pages] int32, row stride bt_stride
  long long bt_stride;
  int page, num_blocks;
  // pieces: positions [pos0, pos0 + count) of request `req` (seq_len cached tokens), written from row `out_row`
  int num_pieces;
  int piece_req[kVarlenMax], piece_len[kVarlenMax], piece_pos0[kVarlenMax], piece_count[kVarlenMax];
  long long piece_out[kVarlenMax];
  int piece_cta0[kVarlenMax + 1];   // first CTA (grid x) of every piece, and the total
  int k_nch[4];
  int k_chunk[4][kPwMaxChunks];
  int v_chunk0, v_nch, v_offset;
  const __nv_bfloat16* cos_sin;
  int max_pos;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  long long out_st, out_sg;
  int* err;
};
cudaError_t launch_decompress(const DecompressMaps& maps, const DecompressParams& p, cudaStream_t stream);
int decompress_piece_ctas(int pos0, int count);

// Prefill attention (prefill_attn.cu).
struct PrefillAttnMaps {
  CUtensorMap q;   // [ql, H, 256], box {64, 1, 128}
  CUtensorMap k;   // [S, G, 256], box {64, 1, 128}
  CUtensorMap v;
};
struct PrefillAttnParams {
  int H, hpg, causal;
  float scale_log2;
  // pieces: queries [q_row, q_row + ql) at positions q_pos0.. over keys [k_row, k_row + S) at positions k_pos0..;
  // outputs (and LSEs) from row o_row of out / lse, or of out2 / lse2 when to2 is set
  int num_pieces;
  int piece_q_row[kVarlenMax], piece_ql[kVarlenMax], piece_k_row[kVarlenMax], piece_S[kVarlenMax];
  int piece_q_pos0[kVarlenMax], piece_k_pos0[kVarlenMax], piece_o_row[kVarlenMax], piece_to2[kVarlenMax];
  int piece_cta0[kVarlenMax + 1];   // first query tile (grid x) of every piece, and the total
  __nv_bfloat16* out;
  __nv_bfloat16* out2;
  long long out_st, out_sh;
  float* lse;          // [rows, H] (row stride lse_st), may be null
  float* lse2;
  long long lse_st;
  int* err;
};
cudaError_t launch_prefill_attn(const PrefillAttnMaps& maps, const PrefillAttnParams& p, cudaStream_t stream);

// Log-sum-exp fold of a chunk's attention result into a running one (attn_fold.cu), in place:
//   out[dst] = bf16((out[dst] e^(lse[dst] - m) + part[src] e^(plse[src] - m)) / s), lse[dst] = m + log s
// for the rows of every piece (dst_row.., src_row.., rows); a part row with LSE -inf leaves its row unchanged, an out row
// with LSE -inf takes the part row.
struct AttnFoldParams {
  __nv_bfloat16* out;
  long long out_st, out_sh;
  float* lse;
  long long lse_st;
  const __nv_bfloat16* part;
  long long part_st, part_sh;
  const float* plse;
  long long plse_st;
  int H;
  int num_pieces;
  int piece_dst[kVarlenMax], piece_src[kVarlenMax], piece_rows[kVarlenMax];
  int piece_row0[kVarlenMax + 1];   // first grid row of every piece, and the total
};
cudaError_t launch_attn_fold(const AttnFoldParams& p, cudaStream_t stream);

// Element-wise steps around the attention (model_ops.cu).
struct QNormRopeParams {
  const __nv_bfloat16* qg;   // [T, H, >= 256] (the query half of each head's q_gate_proj block)
  long long qg_st, qg_sh;
  int T, H;
  const float* w;            // [256] zero-centred RMSNorm weight
  float eps;
  const __nv_bfloat16* cos_sin;   // [max_pos, rot]
  int max_pos, rot;
  const void* positions;
  int pos_i64;
  __nv_bfloat16* q;
  long long q_st, q_sh;
};
cudaError_t launch_q_norm_rope(const QNormRopeParams& p, cudaStream_t stream);
struct GateMulParams {
  const __nv_bfloat16* attn;
  long long attn_st, attn_sh;
  const __nv_bfloat16* gate;
  long long gate_st, gate_sh;
  int T, H;
  __nv_bfloat16* out;
  long long out_st, out_sh;
};
cudaError_t launch_gate_mul(const GateMulParams& p, cudaStream_t stream);

// Dense BF16 GEMM C = A B^T (gemm.cu): maps.a 2-D {K, M} box {64, 128}, maps.b 2-D {K, N} box {64, bn}, both with
// the 128-byte swizzle; tiles of 128 x bn taken round-robin by a persistent grid.
struct GemmMaps {
  CUtensorMap a;
  CUtensorMap b;
};
struct GemmParams {
  __nv_bfloat16* c;
  long long ldc;
  int M, N, K;
  int bn;                       // 128 or 256
  int tiles_m, num_tiles;
  int vec_out;                  // C rows 16-byte aligned
  int stages;                   // set by the launcher
  int* err;
};
cudaError_t launch_gemm(const GemmMaps& maps, GemmParams p, int num_sms, cudaStream_t stream);

// Bounded-wait self-test (selftest.cu).
cudaError_t launch_selftest_wait(int* err, int* status, cudaStream_t stream);

// Launches `kernel` so that it may start while the kernel ahead of it in `stream` is still running (programmatic
// dependent launch): it must call grid_dependency_wait() before it reads anything that kernel writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_after(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                         Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Sets the text belt_last_error() returns on the calling thread.
void set_last_error(const char* msg);

}  // namespace belt
