/*
 * belt_b200 — C ABI of the B200 (sm_100a) latent-KV decode path.
 *
 * Every entry point takes plain device pointers, element strides and sizes, launches on the given CUDA stream
 * (a cudaStream_t passed as void*, NULL = the legacy default stream), allocates nothing and returns
 * BELT_OK or a negative status; belt_last_error() then describes the failure (thread-local). Launches are
 * asynchronous. The launches of the entry points that take every buffer from the caller can be captured in CUDA
 * graphs. BF16 tensors are passed as `const void*` / `void*`.
 *
 * Each entry point but belt_latent_decode_noalloc replaces one operator of the reference's vLLM plugin
 * (liuyaoyang04/BELT, plugins/vllm_lrkv/vllm_lrkv/), cited per function.
 */
#ifndef BELT_B200_H_
#define BELT_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BELT_OK 0
#define BELT_ERR_INVALID (-1)     /* bad shape, stride, alignment or unsupported layout */
#define BELT_ERR_CUDA (-2)        /* a CUDA runtime / driver call failed */

/* Tokens per split-KV tile of the decode kernel (the schedule's unit). */
#define BELT_DECODE_TILE 128

/* Thread-local description of the last failure of a belt_* call on this thread ("" if none). */
const char* belt_last_error(void);

/* ABI version of this library (major * 100 + minor). 200: the per-head GEMM entry points take an error word;
 * 201: belt_path_counts; 202: belt_decode_schedule_balanced, belt_latent_decode_timed. */
int belt_abi_version(void);

/*
 * Host-side counts, since the library was loaded, of the launches that ran a CUDA-core kernel because TMA could not
 * describe the operands (no counterpart in the reference): counts[0] = belt_block_diag_query / belt_up_project calls
 * that took the SIMT group GEMM (strides not multiples of 16 bytes, a misaligned base), counts[1] =
 * belt_latent_rows_to_cache calls that took the SIMT cache write (a group over more than five 64-column chunks, a
 * misaligned u_cat). Writes min(n, 2) counts. The results are the same either way; the counts say which path ran.
 */
int belt_path_counts(int64_t* counts, int32_t n);

/*
 * Split-KV schedule of one decode step: replaces cute_decode.py:601-607 (`schedule`) / :571-598 (`_schedule`).
 * seq_lens [num_reqs] int32 (device, including this step's token) -> work [work_capacity, 4] int32
 * (request, first tile, end tile, 0) per segment, cta_seg [num_ctas + 1] int32, seg_base [num_reqs + 1] int32.
 * Tiles are BELT_DECODE_TILE tokens; runs of max(ceil(tiles / num_ctas), min_tiles) tiles per CTA. A request of
 * length 0 gets no segment. work_capacity >= num_reqs + num_ctas always suffices. err: optional device int32
 * word that receives a nonzero code if the capacity is exceeded.
 */
int belt_decode_schedule(const int32_t* seq_lens, int32_t num_reqs, int32_t num_ctas, int32_t min_tiles,
                         int32_t* work, int64_t work_capacity, int32_t* cta_seg, int32_t* seg_base, int32_t* err,
                         void* stream);

/*
 * The cost-weighted variant of belt_decode_schedule (no reference counterpart; same outputs and capacities): a tile
 * costs 8 units and every request's first tile start_cost (0..1024) more, and the CTAs get equal runs of cost
 * (max(ceil(total / num_ctas), 8 * min_tiles, 8) units) instead of equal runs of tiles. A CTA that switches between
 * requests pays a query reload and a partial-output epilogue per switch in the decode kernel; charging start_cost
 * (about one tile, 8) per request start gives such CTAs fewer tiles, so that the CTAs finish together.
 */
int belt_decode_schedule_weighted(const int32_t* seq_lens, int32_t num_reqs, int32_t num_ctas, int32_t min_tiles,
                                  int32_t start_cost, int32_t* work, int64_t work_capacity, int32_t* cta_seg,
                                  int32_t* seg_base, int32_t* err, void* stream);

/*
 * The weighted split dealt out by measured CTA speed (no reference counterpart; same outputs and capacities as
 * belt_decode_schedule_weighted). cta_ns [num_ctas] int64: per CTA the nanoseconds its decode launches of the previous
 * step took (belt_latent_decode_timed adds them; this call reads and zeroes them); cta_weight [num_ctas] fp32 (start
 * at 1.0): per CTA speed weight, updated in place when every CTA has a time; cta_cap [num_ctas] int64 (written): the
 * cost each CTA was dealt. The update: rate_c = cap_c / ns_c, w_c = clamp(0.5 w_c + 0.5 rate_c / mean(rate),
 * 0.8, 1.25), then normalised to mean 1; CTA c gets the cost range [per * num_ctas * W_c / W, per * num_ctas *
 * W_(c+1) / W) where W_c is the sum of the weights before c (exactly the weighted split when every weight is equal).
 * CTAs on slower SMs get less work, so that the CTAs of a launch finish together. The weights are used only when
 * every CTA gets at least 8 tiles' cost (and num_ctas <= 1024); otherwise this is the weighted split. The split then
 * depends on measured times: two runs of the same step can cut segments at other tiles (results differ at the
 * rounding level of the merge).
 */
int belt_decode_schedule_balanced(const int32_t* seq_lens, int32_t num_reqs, int32_t num_ctas, int32_t min_tiles,
                                  int32_t start_cost, int64_t* cta_ns, float* cta_weight, int64_t* cta_cap,
                                  int32_t* work, int64_t work_capacity, int32_t* cta_seg, int32_t* seg_base,
                                  int32_t* err, void* stream);

/*
 * Absorbed block-diagonal decode query: replaces latent_ops.py:67-73 (`block_diag_query`, the grouped GEMM of
 * :23-44). q [T, 24, 256] BF16 (element strides q_st, q_sh; last dim contiguous) x qmap [4, 256, kq] BF16
 * (contiguous) -> q_bd [T, 24, kq] BF16 (contiguous). Only the columns listed in col_runs are computed for each
 * group (host array [4][3][2] of [start, end) runs, an empty run has start == end); the other columns are written
 * as zeros. A qmap made by `derive_latent_tensors` is zero outside its group's latent columns and RoPE chunk, so
 * passing those runs gives the dense product. err: optional device int32 word that receives a nonzero code if a
 * bounded wait in the tensor-core kernel timed out (the output is then not valid).
 */
int belt_block_diag_query(const void* q, int64_t num_tokens, int64_t q_st, int64_t q_sh, const void* qmap,
                          int32_t kq, const int32_t* col_runs, void* q_bd, int32_t* err, void* stream);

/*
 * Per-head V up-projection: replaces latent_ops.py:76-81 (`up_project`). a [T, 24, r_v] BF16 (strides a_st,
 * a_sh) x v_up_t [4, r_v, 256] BF16 (contiguous, U_v transposed) -> out [T, 24, 256] BF16 (strides out_st, out_sh),
 * written in place (e.g. a view of the first rows of the attention output). err: as belt_block_diag_query.
 */
int belt_up_project(const void* a, int64_t num_tokens, int64_t a_st, int64_t a_sh, int32_t r_v, const void* v_up_t,
                    void* out, int64_t out_st, int64_t out_sh, int32_t* err, void* stream);

/*
 * Latent cache write: replaces latent_ops.py:138-158 (`latent_rows_to_cache`, kernel `_latent_rows` :85-135).
 * c [T, >= W] BF16 (row stride c_st): the latent projection of the new tokens, [c_K | 0 | c_v | 0].
 * slots [T] int32 (slots_i64 = 0) or int64 (slots_i64 = 1); slot s goes to block s / page, row s % page;
 * s < 0 or s >= num_blocks * page is skipped. cache: the layer's [num_blocks, page, W] BF16 view with element
 * strides (stride_block, stride_tok, 1). u_cat [lk, 4 * 256] BF16 contiguous; k_segs: host int32 [4][4] =
 * (start, length, start, length) per group; eps of the k_norm RMS. Writes rows [c_K / rho | c[lk:W]].
 * The RMS fold runs on the tensor cores whenever every group lies within five 64-column chunks and u_cat is 16-byte
 * aligned (a SIMT kernel otherwise); the results agree within one BF16 ulp either way.
 */
int belt_latent_rows_to_cache(const void* c, int64_t num_tokens, int64_t c_st, const void* slots, int32_t slots_i64,
                              void* cache, int64_t num_blocks, int32_t page, int32_t row_width, int64_t stride_block,
                              int64_t stride_tok, const void* u_cat, int32_t lk, const int32_t* k_segs, float eps,
                              void* stream);

/*
 * Fused latent cache write with the down-projection: replaces the model's `kv_latent_proj` linear
 * (models/qwen3_5_latent.py:139-140, 213; weight rows laid out by lrkv/runtime/export_latent.py:193-205) followed by
 * latent_ops.py:138-158 (`latent_rows_to_cache`). x [T, hidden] BF16 (row stride x_st) are the layer's inputs of the
 * new tokens; w_down [>= row_width, hidden] BF16 (row stride w_st) is `kv_latent_proj.weight` (zero rows at the gaps).
 * c = bf16(x w_down^T) is never stored: the kernel writes rows [c_K / rho | c[lk:W]] at slots as
 * belt_latent_rows_to_cache does with that c. hidden, x_st and w_st multiples of 8, x / w_down / u_cat 16-byte
 * aligned. Every group's runs must fit in five 64-column chunks (always true for ranks <= 256). err: optional device
 * word for a wait that timed out.
 */
int belt_latent_proj_rows_to_cache(const void* x, int64_t num_tokens, int64_t x_st, int32_t hidden,
                                   const void* w_down, int64_t w_st, const void* slots, int32_t slots_i64,
                                   void* cache, int64_t num_blocks, int32_t page, int32_t row_width,
                                   int64_t stride_block, int64_t stride_tok, const void* u_cat, int32_t lk,
                                   const int32_t* k_segs, float eps, int32_t* err, void* stream);

/*
 * Single-pass paged latent decode (split-KV partials): replaces cute_decode.py:649-678 (`latent_decode_cute`,
 * kernel `LatentDecodeSm90` :90-484).
 *   q_bd [num_reqs, 24, kq] BF16 contiguous (belt_block_diag_query), kq = n_k * 64 + 4 * 64, n_k = ceil(lk_pad / 64);
 *   cache [num_blocks, page, W] BF16 view, element strides (stride_block, stride_tok, 1), 16-byte aligned rows;
 *     page in {16, 32, 64} or a multiple of 128;
 *   block_table [num_reqs, >= pages] int32 (row stride bt_stride); seq_lens [num_reqs] int32 (this step's token
 *     included, already written);
 *   work / cta_seg: belt_decode_schedule output for these seq_lens with num_ctas CTAs;
 *   part [>= segments, 24, lv + 1] fp32 (element strides part_ss, part_sh; last dim contiguous): per segment the
 *     normalised latent V-space output and the natural-log LSE of the scaled scores;
 *   sm_scale: softmax scale (head_dim^-0.5); lk_pad = v_offset (start of the V part), lv = r_v (<= 640);
 *   rope_groups: host int32 [4][2] = (first column, rr_g) of every group's RoPE coordinates;
 *   rope_blocks [64, n_rope_blocks * 64] BF16 contiguous (`rope_blocks`, cute_decode.py:635-646);
 *   cos_sin [max_pos, 64] BF16 contiguous (cos half | sin half); token t of a request sits at position t;
 *   err: optional device int32 word receiving a nonzero code if a wait in the kernel timed out.
 */
int belt_latent_decode(const void* q_bd, int32_t num_reqs, int32_t kq, const void* cache, int64_t num_blocks,
                       int32_t page, int32_t row_width, int64_t stride_block, int64_t stride_tok,
                       const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens, const int32_t* work,
                       const int32_t* cta_seg, int32_t num_ctas, float* part, int64_t part_ss, int64_t part_sh,
                       float sm_scale, int32_t lk_pad, int32_t lv, const int32_t* rope_groups,
                       const void* rope_blocks, int32_t n_rope_blocks, const void* cos_sin, int32_t max_pos,
                       int32_t* err, void* stream);

/*
 * belt_latent_decode that also times every CTA (no reference counterpart): cta_ns [num_ctas] int64 (device), CTA c
 * adds the nanoseconds from the completion of the kernel ahead of it in the stream (the absorbed query) to its exit.
 * belt_decode_schedule_balanced reads them for the next step's split.
 */
int belt_latent_decode_timed(const void* q_bd, int32_t num_reqs, int32_t kq, const void* cache, int64_t num_blocks,
                             int32_t page, int32_t row_width, int64_t stride_block, int64_t stride_tok,
                             const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                             const int32_t* work, const int32_t* cta_seg, int32_t num_ctas, float* part,
                             int64_t part_ss, int64_t part_sh, float sm_scale, int32_t lk_pad, int32_t lv,
                             const int32_t* rope_groups, const void* rope_blocks, int32_t n_rope_blocks,
                             const void* cos_sin, int32_t max_pos, int32_t* err, int64_t* cta_ns, void* stream);

/*
 * Segment merge: replaces cute_decode.py:715-722 (`merge_segments`, kernel `_merge_segments` :681-712).
 * part [segments, nh, lv + 1] fp32 (strides part_ss, part_sh), seg_base [num_reqs + 1] int32 ->
 * out [num_reqs, nh, lv] BF16 (strides out_sb, out_sh), lse [num_reqs, nh] fp32 (row stride lse_sb).
 * A request without segments gets zeros and -inf.
 */
int belt_merge_segments(const float* part, int64_t part_ss, int64_t part_sh, const int32_t* seg_base,
                        int32_t num_reqs, int32_t nh, int32_t lv, void* out, int64_t out_sb, int64_t out_sh,
                        float* lse, int64_t lse_sb, void* stream);

/*
 * Segment merge and V up-projection in one kernel: belt_merge_segments followed by belt_up_project (cute_decode.py:
 * 715-722 `merge_segments`, then latent_ops.py:76-81 `up_project`), with the merged latent output kept on chip.
 * part [segments, 24, lv + 1] fp32 (strides part_ss, part_sh; last dim contiguous), seg_base [num_reqs + 1] int32,
 * v_up_t [4, lv, 256] BF16 contiguous (U_v transposed) -> out [num_reqs, 24, 256] BF16 (strides out_st, out_sh, 1),
 * lse [num_reqs, 24] fp32 (row stride lse_sb; may be NULL). The merged output is rounded to BF16 before the
 * projection, as the two-kernel path does; lv <= 640. err: optional device error word.
 */
int belt_merge_up_project(const float* part, int64_t part_ss, int64_t part_sh, const int32_t* seg_base,
                          int32_t num_reqs, int32_t lv, const void* v_up_t, void* out, int64_t out_st, int64_t out_sh,
                          float* lse, int64_t lse_sb, int32_t* err, void* stream);

/*
 * One decode step of a compressed layer with no caller-provided scratch: belt_decode_schedule_weighted (start cost
 * 13, the backend's start cost; no speed balancing, which needs state across steps), belt_latent_decode and belt_merge_segments in a row on `stream`, with the segment records and split-KV partials kept in a fixed
 * 24 MiB array inside this library instead of buffers from the caller. It has no counterpart in the reference
 * (whose decode allocates its partials per call); it exists for callers that cannot allocate device memory: hosts
 * binding this ABI that hold only the engine's KV pool, query and output buffers, and engines that reserved nearly
 * all of HBM for the KV pool at start-up. It calls no allocating routine.
 *   Arguments as belt_latent_decode, minus work / cta_seg / part, plus min_tiles (belt_decode_schedule) and the
 *   merged outputs out [num_reqs, 24, lv] BF16 (strides out_sb, out_sh) and lse [num_reqs, 24] fp32 (row stride
 *   lse_sb), as belt_merge_segments. Pointers and `stream` belong to the current device.
 *   Limits (BELT_ERR_INVALID beyond them, before anything runs): num_reqs <= 4096, num_ctas <= 1024, and
 *   (num_reqs + num_ctas) * 24 * (lv + 1) * 4 bytes <= 24 MiB - 128 KiB (lv = 640, 148 CTAs: 258 requests).
 *   The array's device address belongs to the CUDA context: a call outside stream capture looks it up
 *   (cudaGetSymbolAddress) and records it for the current context; a call during capture uses that record and is
 *   refused if the context has none. Make the first call in a context (a device's first, the first under a
 *   driver-API context, the first after cudaDeviceReset) before any stream capture begins. All calls on a device
 *   share the array and leave their contents in it; calls that overlap on the GPU (unordered streams or host threads
 *   of one device) race on it.
 */
int belt_latent_decode_noalloc(const void* q_bd, int32_t num_reqs, int32_t kq, const void* cache, int64_t num_blocks,
                               int32_t page, int32_t row_width, int64_t stride_block, int64_t stride_tok,
                               const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                               int32_t num_ctas, int32_t min_tiles, float sm_scale, int32_t lk_pad, int32_t lv,
                               const int32_t* rope_groups, const void* rope_blocks, int32_t n_rope_blocks,
                               const void* cos_sin, int32_t max_pos, void* out, int64_t out_sb, int64_t out_sh,
                               float* lse, int64_t lse_sb, int32_t* err, void* stream);

/*
 * Keys and values of cached positions [pos0, pos0 + count) of one request, rebuilt from its latent rows: replaces
 * latent_backend.py:95-108 (`LatentLayer.decompress`) applied to rows gathered through the request's block table
 * (latent_backend.py:214-225), the prefill path's input to its attention.
 *   cache [num_blocks, page, W] BF16 view as belt_latent_decode; block_table_row [>= ceil(seq_len / page)] int32;
 *   wk [4, 256, kc] BF16 contiguous: per group [rope_up[g]; qmap[g, 64:, :kc]], kc = n_k * 64;
 *   k_segs host int32 [4][4] (the groups' column runs); v_up [4, r_v, 256] BF16 contiguous; cos_sin [max_pos, 64];
 *   k_out, v_out [count, 4, 256] BF16 views with element strides (out_st, out_sg, 1): k = [RoPE(bf16(x)) | k_nope].
 * Rounding as the reference: BF16 products of the matmuls, the rotation in fp32, BF16 out.
 */
int belt_latent_decompress(const void* cache, int64_t num_blocks, int32_t page, int32_t row_width,
                           int64_t stride_block, int64_t stride_tok, const int32_t* block_table_row, int32_t seq_len,
                           int32_t pos0, int32_t count, const void* wk, int32_t kc, const int32_t* k_segs,
                           const void* v_up, int32_t v_offset, int32_t r_v, const void* cos_sin, int32_t max_pos,
                           void* k_out, void* v_out, int64_t out_st, int64_t out_sg, int32_t* err, void* stream);

/*
 * Prefill attention over rebuilt keys and values: replaces the reference's flash_attn_varlen_func call in its
 * prefill path (latent_backend.py:285-320; one request at a time). q [ql, 24, 256] BF16 (element strides q_st, q_sh,
 * 1), k / v [num_keys, 4, 256] BF16 (kv_st, kv_sg, 1; head h reads group h / 6), query i at position q_pos0 + i, key j
 * at k_pos0 + j; causal: key j is seen by query i when its position is not after the query's. out [ql, 24, 256] BF16
 * (out_st, out_sh, 1) = softmax(scale q k^T) v; lse [ql, 24] fp32 (row stride lse_st, may be NULL): the natural-log
 * sum of exp(scale q k^T) over the keys seen, -inf (and a zero output) when a query sees none.
 */
int belt_prefill_attention(const void* q, int32_t ql, int64_t q_st, int64_t q_sh, const void* k, const void* v,
                           int32_t num_keys, int64_t kv_st, int64_t kv_sg, int32_t q_pos0, int32_t k_pos0,
                           int32_t causal, float scale, void* out, int64_t out_st, int64_t out_sh, float* lse,
                           int64_t lse_st, int32_t* err, void* stream);

/*
 * Dense BF16 GEMM on the tensor cores: c[M, N] = a[M, K] b[N, K]^T (both K-major: a row-major with row stride lda, b
 * row-major [N, K] with row stride ldb, the layout of a torch Linear weight), FP32 accumulation, BF16 out (row stride
 * ldc). Replaces the model's linear layers around the latent attention (models/qwen3_5_latent.py:130-140, 204-217:
 * q_gate_proj, o_proj, and kv_latent_proj where the prefill computes the latent rows). K, lda, ldb multiples of 8;
 * a, b 16-byte aligned. err: optional device word for a wait that timed out.
 */
int belt_gemm_bf16(const void* a, int64_t m, int64_t k, int64_t lda, const void* b, int64_t n, int64_t ldb, void* c,
                   int64_t ldc, int32_t* err, void* stream);

/*
 * belt_latent_decompress over several pieces in one launch (the reference decompresses all prefill requests of a step
 * together, latent_backend.py:214-225, 285-320). pieces: host int32 [num_pieces][4] = (request: row of block_table,
 * seq_len, pos0, count); block_table [requests, >= pages] int32 with row stride bt_stride. The keys and values of
 * piece i fill rows [sum of the earlier counts, + count_i) of k_out / v_out. Other arguments as belt_latent_decompress.
 */
int belt_latent_decompress_varlen(const void* cache, int64_t num_blocks, int32_t page, int32_t row_width,
                                  int64_t stride_block, int64_t stride_tok, const int32_t* block_table,
                                  int64_t bt_stride, int32_t num_pieces, const int32_t* pieces, const void* wk,
                                  int32_t kc, const int32_t* k_segs, const void* v_up, int32_t v_offset, int32_t r_v,
                                  const void* cos_sin, int32_t max_pos, void* k_out, void* v_out, int64_t out_st,
                                  int64_t out_sg, int32_t* err, void* stream);

/*
 * belt_prefill_attention over several pieces in one launch: the reference's flash_attn_varlen_func calls over all
 * prefill requests of a step (latent_backend.py:285-320). q [q_rows, 24, 256] and k / v [k_rows, 4, 256] are the
 * concatenated queries and rebuilt keys / values; pieces: host int32 [num_pieces][8] = (q_row, ql, k_row, S, q_pos0,
 * k_pos0, o_row, to2): queries [q_row, q_row + ql) at positions q_pos0.. over keys [k_row, k_row + S) at positions
 * k_pos0.., causal by position; outputs and LSEs from row o_row of out / lse (to2 = 0) or of out2 / lse2 (to2 = 1;
 * same strides). lse / lse2 may be NULL when no piece writes there.
 */
int belt_prefill_attention_varlen(const void* q, int64_t q_rows, int64_t q_st, int64_t q_sh, const void* k,
                                  const void* v, int64_t k_rows, int64_t kv_st, int64_t kv_sg, int32_t num_pieces,
                                  const int32_t* pieces, int32_t causal, float scale, void* out, void* out2,
                                  int64_t out_st, int64_t out_sh, float* lse, float* lse2, int64_t lse_st,
                                  int32_t* err, void* stream);

/*
 * The log-sum-exp fold of one chunk's attention result into the running one, in place: the reference merges every
 * context chunk of its prefill into the output with vLLM's merge_attn_states (latent_backend.py:300-320).
 * out [rows, 24, 256] BF16 (strides out_st, out_sh, 1), lse [rows, 24] fp32 (row stride lse_st); part / part_lse the
 * chunk's output and LSE. pieces: host int32 [num_pieces][3] = (destination row, source row, rows). Per row and head:
 * m = max(lse, plse), out = bf16((out e^(lse - m) + part e^(plse - m)) / (e^(lse - m) + e^(plse - m))),
 * lse = m + log(e^(lse - m) + e^(plse - m)); a part row with LSE -inf leaves the row unchanged, a running row with LSE
 * -inf takes the part row.
 */
int belt_attn_fold(void* out, int64_t out_st, int64_t out_sh, float* lse, int64_t lse_st, const void* part,
                   int64_t part_st, int64_t part_sh, const float* part_lse, int64_t plse_st, int32_t num_pieces,
                   const int32_t* pieces, void* stream);

/*
 * The query side of the model's fused q-norm / RoPE (models/qwen3_5_latent.py:209-212, `fused_qk_rmsnorm_rope_gate`
 * with no key heads): qg [T, 24, >= 256] BF16 (element strides qg_st, qg_sh, 1; the query half of every head's
 * q_gate_proj block) -> q [T, 24, 256] BF16 = NeoX rotation of the first `rot` channels (BF16 cos / sin table
 * [max_pos, rot], cos then sin) of x * rsqrt(mean(x^2) + eps) * (1 + norm_weight) (fp32, zero-centred RMSNorm weight
 * [256] fp32), rounded to BF16 once. positions [T] int32 or int64 (positions_i64).
 */
int belt_q_norm_rope(const void* qg, int32_t num_tokens, int64_t qg_st, int64_t qg_sh, const float* norm_weight,
                     float eps, const void* cos_sin, int32_t max_pos, int32_t rot, const void* positions,
                     int32_t positions_i64, void* q, int64_t q_st, int64_t q_sh, void* stream);

/*
 * The output gate (models/qwen3_5_latent.py:215): out = attn * sigmoid(gate), all [T, 24, 256] BF16 views with
 * element strides (st, sh, 1); out may alias attn.
 */
int belt_gate_mul(const void* attn, int64_t attn_st, int64_t attn_sh, const void* gate, int64_t gate_st,
                  int64_t gate_sh, int32_t num_tokens, void* out, int64_t out_st, int64_t out_sh, void* stream);

/*
 * Self-test of the kernels' bounded waits (no counterpart in the reference): launches one thread that waits on a
 * barrier nothing completes. The wait gives up after the same limit the decode kernel uses (~2 s), writes 0x1F0 into
 * the device word `err` (if still 0), and the kernel ends normally; status (device int32[2]) receives {2, 1} (wait gave
 * up, abort flag raised). For tests of failure detection: the CUDA context stays usable afterwards.
 */
int belt_selftest_bounded_wait(int32_t* err, int32_t* status, void* stream);

/* Number of SMs of `device` (the decode grid: one CTA per SM). */
int belt_num_sms(int32_t device);

#ifdef __cplusplus
}
#endif

#endif /* BELT_B200_H_ */
