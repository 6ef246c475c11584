// The C ABI (include/belt_b200.h): argument checks, TMA descriptor encoding and kernel launches.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/belt_b200.h"
#include "common.cuh"
#include "launch.h"

namespace {

thread_local std::string g_last_error;

// Launches that took a CUDA-core kernel because TMA could not describe the operands (see belt_path_counts).
std::atomic<long long> g_simt_group_gemm{0};
std::atomic<long long> g_simt_cache_write{0};

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(BELT_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int ok() {
  g_last_error.clear();
  return BELT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// BF16 tiled map with 128-byte swizzle; dims / strides innermost first (strides in bytes, rank - 1 of them).
int encode_bf16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                const cuuint32_t* box, const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(BELT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BELT_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", what, (int)r);
  return BELT_OK;
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Out = X W per head's group (block_diag_query, up_project): on the tensor cores when TMA can describe X and W
// (16-byte aligned bases and strides, W rows contiguous), else on the SIMT kernel.
int run_group_product(const belt::GroupGemmParams& gp, const char* what, int32_t* err, cudaStream_t stream) {
  const bool tma_ok = aligned16(gp.X) && aligned16(gp.W) && gp.swn == 1 && gp.sxh > 0 && gp.sxt > 0 &&
                      (gp.sxh * 2) % 16 == 0 && (gp.sxt * 2) % 16 == 0 && (gp.swk * 2) % 16 == 0 &&
                      (gp.swg * 2) % 16 == 0 && gp.K > 0 && gp.sxh >= gp.K &&
                      gp.sxt >= static_cast<long long>(gp.G * gp.hpg) * gp.sxh && gp.swk >= gp.N &&
                      gp.swg >= static_cast<long long>(gp.K) * gp.swk;
  cudaError_t e;
  if (tma_ok) {
    belt::HeadGemmMaps maps;
    {
      cuuint64_t dims[3] = {static_cast<cuuint64_t>(gp.K), static_cast<cuuint64_t>(gp.G * gp.hpg),
                            static_cast<cuuint64_t>(gp.T)};
      cuuint64_t strides[2] = {static_cast<cuuint64_t>(gp.sxh) * 2, static_cast<cuuint64_t>(gp.sxt) * 2};
      cuuint32_t box[3] = {64, 1, 128};
      int r = encode_bf16(&maps.x, gp.X, 3, dims, strides, box, what);
      if (r != BELT_OK) return r;
    }
    {
      cuuint64_t dims[3] = {static_cast<cuuint64_t>(gp.N), static_cast<cuuint64_t>(gp.K),
                            static_cast<cuuint64_t>(gp.G)};
      cuuint64_t strides[2] = {static_cast<cuuint64_t>(gp.swk) * 2, static_cast<cuuint64_t>(gp.swg) * 2};
      cuuint32_t box[3] = {64, 64, 1};
      int r = encode_bf16(&maps.w, gp.W, 3, dims, strides, box, what);
      if (r != BELT_OK) return r;
    }
    belt::HeadGemmParams hp{};
    hp.Out = gp.Out;
    hp.sot = gp.sot;
    hp.soh = gp.soh;
    hp.T = gp.T;
    hp.K = gp.K;
    hp.N = gp.N;
    hp.hpg = gp.hpg;
    hp.G = gp.G;
    for (int g = 0; g < 4; ++g) {
      hp.nruns[g] = gp.nruns[g];
      for (int i = 0; i < 3; ++i) {
        hp.run_lo[g][i] = gp.run_lo[g][i];
        hp.run_hi[g][i] = gp.run_hi[g][i];
      }
    }
    // column tile: 128 columns for the wide absorbed query (most tiles are outside the runs and only write zeros),
    // 64 for the 256-column U_v projection (more CTAs for its deeper K loop)
    hp.nb = gp.N <= 256 ? 1 : 2;
    hp.vec_out = aligned16(gp.Out) && gp.sot % 8 == 0 && gp.soh % 8 == 0;
    hp.err = err;
    e = belt::launch_head_gemm(maps, hp, stream);
  } else {
    e = belt::launch_group_gemm(gp, stream);
    g_simt_group_gemm.fetch_add(1, std::memory_order_relaxed);
  }
  if (e != cudaSuccess) {
    char buf[96];
    snprintf(buf, sizeof(buf), "%s launch", what);
    return cuda_fail(e, buf);
  }
  return BELT_OK;
}

}  // namespace

void belt::set_last_error(const char* msg) { g_last_error = msg; }

extern "C" {

const char* belt_last_error(void) { return g_last_error.c_str(); }

int belt_abi_version(void) { return 202; }

int belt_path_counts(int64_t* counts, int32_t n) {
  if (!counts || n < 0) return fail(BELT_ERR_INVALID, "path_counts: null buffer");
  const long long v[2] = {g_simt_group_gemm.load(std::memory_order_relaxed),
                          g_simt_cache_write.load(std::memory_order_relaxed)};
  for (int i = 0; i < n && i < 2; ++i) counts[i] = v[i];
  return ok();
}

int belt_num_sms(int32_t device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  return n;
}

int belt_decode_schedule(const int32_t* seq_lens, int32_t num_reqs, int32_t num_ctas, int32_t min_tiles,
                         int32_t* work, int64_t work_capacity, int32_t* cta_seg, int32_t* seg_base, int32_t* err,
                         void* stream) {
  if (num_reqs < 0 || num_ctas < 1) return fail(BELT_ERR_INVALID, "schedule: num_reqs %d, num_ctas %d", num_reqs, num_ctas);
  if ((num_reqs > 0 && !seq_lens) || !work || !cta_seg || !seg_base)
    return fail(BELT_ERR_INVALID, "schedule: null buffer");
  if (work_capacity < static_cast<int64_t>(num_reqs) + num_ctas)
    return fail(BELT_ERR_INVALID, "schedule: work capacity %lld < num_reqs + num_ctas = %lld",
                (long long)work_capacity, (long long)num_reqs + num_ctas);
  belt::ScheduleParams p{seq_lens, num_reqs, num_ctas, min_tiles, BELT_DECODE_TILE, 1, 0, work, work_capacity,
                         cta_seg, seg_base, err};
  cudaError_t e = belt::launch_schedule(p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "schedule launch");
}

int belt_decode_schedule_weighted(const int32_t* seq_lens, int32_t num_reqs, int32_t num_ctas, int32_t min_tiles,
                                  int32_t start_cost, int32_t* work, int64_t work_capacity, int32_t* cta_seg,
                                  int32_t* seg_base, int32_t* err, void* stream) {
  if (num_reqs < 0 || num_ctas < 1) return fail(BELT_ERR_INVALID, "schedule: num_reqs %d, num_ctas %d", num_reqs, num_ctas);
  if (start_cost < 0 || start_cost > 1024) return fail(BELT_ERR_INVALID, "schedule: start_cost %d outside [0, 1024]", start_cost);
  if ((num_reqs > 0 && !seq_lens) || !work || !cta_seg || !seg_base)
    return fail(BELT_ERR_INVALID, "schedule: null buffer");
  if (work_capacity < static_cast<int64_t>(num_reqs) + num_ctas)
    return fail(BELT_ERR_INVALID, "schedule: work capacity %lld < num_reqs + num_ctas = %lld",
                (long long)work_capacity, (long long)num_reqs + num_ctas);
  belt::ScheduleParams p{seq_lens, num_reqs, num_ctas, min_tiles, BELT_DECODE_TILE, 8, start_cost, work,
                         work_capacity, cta_seg, seg_base, err};
  cudaError_t e = belt::launch_schedule(p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "schedule launch");
}

int belt_decode_schedule_balanced(const int32_t* seq_lens, int32_t num_reqs, int32_t num_ctas, int32_t min_tiles,
                                  int32_t start_cost, int64_t* cta_ns, float* cta_weight, int64_t* cta_cap,
                                  int32_t* work, int64_t work_capacity, int32_t* cta_seg, int32_t* seg_base,
                                  int32_t* err, void* stream) {
  if (num_reqs < 0 || num_ctas < 1) return fail(BELT_ERR_INVALID, "schedule: num_reqs %d, num_ctas %d", num_reqs, num_ctas);
  if (start_cost < 0 || start_cost > 1024) return fail(BELT_ERR_INVALID, "schedule: start_cost %d outside [0, 1024]", start_cost);
  if ((num_reqs > 0 && !seq_lens) || !work || !cta_seg || !seg_base || !cta_ns || !cta_weight || !cta_cap)
    return fail(BELT_ERR_INVALID, "schedule: null buffer");
  if (work_capacity < static_cast<int64_t>(num_reqs) + num_ctas)
    return fail(BELT_ERR_INVALID, "schedule: work capacity %lld < num_reqs + num_ctas = %lld",
                (long long)work_capacity, (long long)num_reqs + num_ctas);
  belt::ScheduleParams p{seq_lens, num_reqs, num_ctas, min_tiles, BELT_DECODE_TILE, 8, start_cost, work,
                         work_capacity, cta_seg, seg_base, err, reinterpret_cast<long long*>(cta_ns), cta_weight,
                         reinterpret_cast<long long*>(cta_cap)};
  cudaError_t e = belt::launch_schedule(p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "schedule launch");
}

int belt_block_diag_query(const void* q, int64_t num_tokens, int64_t q_st, int64_t q_sh, const void* qmap,
                          int32_t kq, const int32_t* col_runs, void* q_bd, int32_t* err, void* stream) {
  if (num_tokens < 0 || kq <= 0 || !col_runs) return fail(BELT_ERR_INVALID, "block_diag_query: bad arguments");
  if (num_tokens == 0) return ok();
  if (!q || !qmap || !q_bd) return fail(BELT_ERR_INVALID, "block_diag_query: null buffer");
  belt::GroupGemmParams p{};
  p.X = static_cast<const __nv_bfloat16*>(q);
  p.sxt = q_st;
  p.sxh = q_sh;
  p.W = static_cast<const __nv_bfloat16*>(qmap);
  p.swg = static_cast<long long>(belt::kD) * kq;
  p.swk = kq;
  p.swn = 1;
  p.Out = static_cast<__nv_bfloat16*>(q_bd);
  p.sot = static_cast<long long>(belt::kH) * kq;
  p.soh = kq;
  p.T = static_cast<int>(num_tokens);
  p.K = belt::kD;
  p.N = kq;
  p.hpg = belt::kHPG;
  p.G = belt::kG;
  for (int g = 0; g < belt::kG; ++g) {
    p.nruns[g] = 3;
    for (int i = 0; i < 3; ++i) {
      const int lo = col_runs[(g * 3 + i) * 2], hi = col_runs[(g * 3 + i) * 2 + 1];
      if (lo < 0 || hi < lo || hi > kq) return fail(BELT_ERR_INVALID, "block_diag_query: column run [%d, %d) of group %d", lo, hi, g);
      p.run_lo[g][i] = lo;
      p.run_hi[g][i] = hi;
    }
  }
  const int r = run_group_product(p, "block_diag_query", err, as_stream(stream));
  return r == BELT_OK ? ok() : r;
}

int belt_up_project(const void* a, int64_t num_tokens, int64_t a_st, int64_t a_sh, int32_t r_v, const void* v_up_t,
                    void* out, int64_t out_st, int64_t out_sh, int32_t* err, void* stream) {
  if (num_tokens < 0 || r_v <= 0) return fail(BELT_ERR_INVALID, "up_project: bad arguments");
  if (num_tokens == 0) return ok();
  if (!a || !v_up_t || !out) return fail(BELT_ERR_INVALID, "up_project: null buffer");
  belt::GroupGemmParams p{};
  p.X = static_cast<const __nv_bfloat16*>(a);
  p.sxt = a_st;
  p.sxh = a_sh;
  p.W = static_cast<const __nv_bfloat16*>(v_up_t);
  p.swg = static_cast<long long>(r_v) * belt::kD;
  p.swk = belt::kD;
  p.swn = 1;
  p.Out = static_cast<__nv_bfloat16*>(out);
  p.sot = out_st;
  p.soh = out_sh;
  p.T = static_cast<int>(num_tokens);
  p.K = r_v;
  p.N = belt::kD;
  p.hpg = belt::kHPG;
  p.G = belt::kG;
  for (int g = 0; g < belt::kG; ++g) {
    p.nruns[g] = 1;
    p.run_lo[g][0] = 0;
    p.run_hi[g][0] = belt::kD;
  }
  const int r = run_group_product(p, "up_project", err, as_stream(stream));
  return r == BELT_OK ? ok() : r;
}

// Work items of the fused write (proj_write.cu) for a row layout: every group's 64-column window, then the V part
// [lk, W) in windows of two chunks; also the groups' runs. Returns BELT_OK or fails with `who` in the message.
static int pw_items(belt::ProjWriteParams& p, const int32_t* k_segs, int32_t lk, int32_t row_width, const char* who) {
  int items = 0;
  for (int g = 0; g < belt::kG; ++g) {
    p.a_lo[g] = k_segs[4 * g];
    p.a_n[g] = k_segs[4 * g + 1];
    p.b_lo[g] = k_segs[4 * g + 2];
    p.b_n[g] = k_segs[4 * g + 3];
    const int r = p.a_n[g] + p.b_n[g];
    if (p.a_lo[g] < 0 || p.b_lo[g] < 0 || p.a_n[g] < 0 || p.b_n[g] < 0 || r > 256 ||
        p.a_lo[g] + p.a_n[g] > lk || (p.b_n[g] > 0 && p.b_lo[g] + p.b_n[g] > lk))
      return fail(BELT_ERR_INVALID, "%s: k_segs of group %d out of range (lk %d)", who, g, lk);
    bool use[64] = {};
    const int runs[2][2] = {{p.a_lo[g], p.a_n[g]}, {p.b_lo[g], p.b_n[g]}};
    for (int q = 0; q < 2; ++q)
      if (runs[q][1] > 0)
        for (int c = runs[q][0] >> 6; c <= (runs[q][0] + runs[q][1] - 1) >> 6 && c < 64; ++c) use[c] = true;
    int n = 0;
    for (int c = 0; c < 64; ++c)
      if (use[c]) {
        if (n == belt::kPwMaxChunks)
          return fail(BELT_ERR_INVALID, "%s: group %d spans more than %d 64-column chunks", who, g,
                      belt::kPwMaxChunks);
        p.item_chunk[items][n++] = c;
      }
    if (n == 0) {   // a group without coordinates still gets an item (nothing to write); keep one chunk to stream
      p.item_chunk[items][0] = 0;
      n = 1;
    }
    p.item_nch[items++] = n;
  }
  // V part in windows of two 64-column chunks: more CTAs, each streaming a smaller share of W_down
  constexpr int kVChunks = 2;
  for (int c = lk >> 6; c < (row_width + 63) >> 6; c += kVChunks) {
    if (items == belt::kPwMaxItems)
      return fail(BELT_ERR_INVALID, "%s: V part too wide (%d columns)", who, row_width - lk);
    const int n = ((row_width + 63) >> 6) - c < kVChunks ? ((row_width + 63) >> 6) - c : kVChunks;
    for (int i = 0; i < n; ++i) p.item_chunk[items][i] = c + i;
    p.item_nch[items++] = n;
  }
  p.n_items = items;
  return BELT_OK;
}

int belt_latent_rows_to_cache(const void* c, int64_t num_tokens, int64_t c_st, const void* slots, int32_t slots_i64,
                              void* cache, int64_t num_blocks, int32_t page, int32_t row_width, int64_t stride_block,
                              int64_t stride_tok, const void* u_cat, int32_t lk, const int32_t* k_segs, float eps,
                              void* stream) {
  if (num_tokens < 0 || page <= 0 || row_width <= 0 || lk < 0 || lk > row_width || !k_segs || num_blocks < 0)
    return fail(BELT_ERR_INVALID, "latent_rows_to_cache: bad arguments");
  if (num_tokens == 0) return ok();
  if (!c || !slots || !cache || !u_cat) return fail(BELT_ERR_INVALID, "latent_rows_to_cache: null buffer");
  belt::CacheWriteParams p{};
  p.c = static_cast<const __nv_bfloat16*>(c);
  p.sct = c_st;
  p.slots = slots;
  p.slots_i64 = slots_i64 ? 1 : 0;
  p.cache = static_cast<__nv_bfloat16*>(cache);
  p.sblk = stride_block;
  p.stok = stride_tok;
  p.page = page;
  p.W = row_width;
  p.lk = lk;
  p.T = static_cast<int>(num_tokens);
  p.G = belt::kG;
  p.num_slots = num_blocks * page;
  p.u_cat = static_cast<const __nv_bfloat16*>(u_cat);
  p.eps = eps;
  for (int g = 0; g < belt::kG; ++g) {
    p.a_lo[g] = k_segs[4 * g];
    p.a_n[g] = k_segs[4 * g + 1];
    p.b_lo[g] = k_segs[4 * g + 2];
    p.b_n[g] = k_segs[4 * g + 3];
    const int r = p.a_n[g] + p.b_n[g];
    if (p.a_lo[g] < 0 || p.b_lo[g] < 0 || p.a_n[g] < 0 || p.b_n[g] < 0 || r > 256 ||
        p.a_lo[g] + p.a_n[g] > lk || (p.b_n[g] > 0 && p.b_lo[g] + p.b_n[g] > lk))
      return fail(BELT_ERR_INVALID, "latent_rows_to_cache: k_segs of group %d out of range (lk %d)", g, lk);
  }
  // The fused write's kernel in c-input mode (RMS fold on the tensor cores) wherever the layout fits it: every group
  // within five 64-column chunks, u_cat 16-byte aligned. Otherwise the SIMT kernel below.
  if (lk > 0 && stride_tok >= row_width && aligned16(u_cat) && num_tokens <= (1ll << 31) - 1) {
    belt::ProjWriteParams q{};
    q.slots = slots;
    q.slots_i64 = slots_i64 ? 1 : 0;
    q.num_slots = num_blocks * page;
    q.cache = static_cast<__nv_bfloat16*>(cache);
    q.sblk = stride_block;
    q.stok = stride_tok;
    q.page = page;
    q.W = row_width;
    q.lk = lk;
    q.T = static_cast<int>(num_tokens);
    q.G = belt::kG;
    q.eps = eps;
    q.vec_ok = aligned16(cache) && stride_tok % 8 == 0 && stride_block % 8 == 0;
    q.c = static_cast<const __nv_bfloat16*>(c);
    q.sct = c_st;
    q.c_in = 1;
    q.c_vec = aligned16(c) && c_st % 8 == 0;
    if (pw_items(q, k_segs, lk, row_width, "latent_rows_to_cache") == BELT_OK) {
      belt::ProjWriteMaps maps{};
      cuuint64_t dims[2] = {static_cast<cuuint64_t>(belt::kG * belt::kD), static_cast<cuuint64_t>(lk)};
      cuuint64_t strides[1] = {static_cast<cuuint64_t>(belt::kG * belt::kD) * 2};
      cuuint32_t box[2] = {64, 64};
      int r = encode_bf16(&maps.u, u_cat, 2, dims, strides, box, "u_cat");
      if (r != BELT_OK) return r;
      cudaError_t e = belt::launch_proj_write(maps, q, as_stream(stream));
      return e == cudaSuccess ? ok() : cuda_fail(e, "latent_rows_to_cache launch");
    }
  }
  g_simt_cache_write.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = belt::launch_cache_write(p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "latent_rows_to_cache launch");
}

int belt_latent_proj_rows_to_cache(const void* x, int64_t num_tokens, int64_t x_st, int32_t hidden,
                                   const void* w_down, int64_t w_st, const void* slots, int32_t slots_i64,
                                   void* cache, int64_t num_blocks, int32_t page, int32_t row_width,
                                   int64_t stride_block, int64_t stride_tok, const void* u_cat, int32_t lk,
                                   const int32_t* k_segs, float eps, int32_t* err, void* stream) {
  if (num_tokens < 0 || page <= 0 || row_width <= 0 || lk <= 0 || lk > row_width || !k_segs || num_blocks < 0 ||
      hidden <= 0)
    return fail(BELT_ERR_INVALID, "latent_proj_rows_to_cache: bad arguments");
  if (num_tokens == 0) return ok();
  if (!x || !w_down || !slots || !cache || !u_cat) return fail(BELT_ERR_INVALID, "latent_proj_rows_to_cache: null buffer");
  if (hidden % 8 || x_st < hidden || x_st % 8 || w_st < hidden || w_st % 8 || !aligned16(x) || !aligned16(w_down) ||
      !aligned16(u_cat))
    return fail(BELT_ERR_INVALID,
                "latent_proj_rows_to_cache: x and W_down need 16-byte aligned rows (hidden %d, strides %lld, %lld)",
                hidden, (long long)x_st, (long long)w_st);
  if (stride_tok < row_width) return fail(BELT_ERR_INVALID, "latent_proj_rows_to_cache: token stride < row width");
  if (num_tokens > (1ll << 31) - 1) return fail(BELT_ERR_INVALID, "latent_proj_rows_to_cache: too many tokens");
  belt::ProjWriteParams p{};
  p.slots = slots;
  p.slots_i64 = slots_i64 ? 1 : 0;
  p.num_slots = num_blocks * page;
  p.cache = static_cast<__nv_bfloat16*>(cache);
  p.sblk = stride_block;
  p.stok = stride_tok;
  p.page = page;
  p.W = row_width;
  p.lk = lk;
  p.T = static_cast<int>(num_tokens);
  p.hidden = hidden;
  p.G = belt::kG;
  p.eps = eps;
  p.vec_ok = aligned16(cache) && stride_tok % 8 == 0 && stride_block % 8 == 0;
  p.err = err;
  {
    const int r = pw_items(p, k_segs, lk, row_width, "latent_proj_rows_to_cache");
    if (r != BELT_OK) return r;
  }
  belt::ProjWriteMaps maps;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(num_tokens)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(x_st) * 2};
    cuuint32_t box[2] = {64, 128};
    int r = encode_bf16(&maps.x, x, 2, dims, strides, box, "x");
    if (r != BELT_OK) return r;
  }
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(row_width)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(w_st) * 2};
    cuuint32_t box[2] = {64, 64};
    int r = encode_bf16(&maps.w, w_down, 2, dims, strides, box, "w_down");
    if (r != BELT_OK) return r;
  }
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(belt::kG * belt::kD), static_cast<cuuint64_t>(lk)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(belt::kG * belt::kD) * 2};
    cuuint32_t box[2] = {64, 64};
    int r = encode_bf16(&maps.u, u_cat, 2, dims, strides, box, "u_cat");
    if (r != BELT_OK) return r;
  }
  cudaError_t e = belt::launch_proj_write(maps, p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "latent_proj_rows_to_cache launch");
}

namespace {
int latent_decode_impl(const void* q_bd, int32_t num_reqs, int32_t kq, const void* cache, int64_t num_blocks,
                       int32_t page, int32_t row_width, int64_t stride_block, int64_t stride_tok,
                       const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens, const int32_t* work,
                       const int32_t* cta_seg, int32_t num_ctas, float* part, int64_t part_ss, int64_t part_sh,
                       float sm_scale, int32_t lk_pad, int32_t lv, const int32_t* rope_groups,
                       const void* rope_blocks, int32_t n_rope_blocks, const void* cos_sin, int32_t max_pos,
                       int32_t* err, int64_t* cta_ns, void* stream) {
  using namespace belt;
  if (num_reqs < 0 || num_ctas < 1) return fail(BELT_ERR_INVALID, "latent_decode: num_reqs %d, num_ctas %d", num_reqs, num_ctas);
  if (num_reqs == 0) return ok();
  if (!q_bd || !cache || !block_table || !seq_lens || !work || !cta_seg || !part || !rope_groups || !rope_blocks ||
      !cos_sin)
    return fail(BELT_ERR_INVALID, "latent_decode: null buffer");
  const int n_k = (lk_pad + 63) / 64;
  if (lk_pad <= 0 || lk_pad % 8 || n_k + kG > kDecodeMaxQChunks)
    return fail(BELT_ERR_INVALID, "latent_decode: lk_pad %d must be a positive multiple of 8 and at most %d", lk_pad,
                (kDecodeMaxQChunks - kG) * 64);
  if (kq != n_k * 64 + kG * kRot) return fail(BELT_ERR_INVALID, "latent_decode: kq %d != n_k * 64 + 256 = %d", kq, n_k * 64 + 256);
  if (lv <= 0 || lv > 128 * kDecodeMaxVPairs) return fail(BELT_ERR_INVALID, "latent_decode: lv %d outside (0, 640]", lv);
  if (lk_pad + lv > row_width) return fail(BELT_ERR_INVALID, "latent_decode: lk_pad + lv %d > row width %d", lk_pad + lv, row_width);
  if (!(page == 16 || page == 32 || page == 64 || (page % 128 == 0 && page > 0)))
    return fail(BELT_ERR_INVALID, "latent_decode: page size %d (supported: 16, 32, 64 or a multiple of 128)", page);
  if (num_blocks < 1 || num_blocks > (1ll << 31) - 2) return fail(BELT_ERR_INVALID, "latent_decode: num_blocks %lld", (long long)num_blocks);
  if (!aligned16(cache) || stride_tok % 8 || stride_block % 8 || stride_tok < row_width)
    return fail(BELT_ERR_INVALID, "latent_decode: cache rows must be 16-byte aligned (strides %lld, %lld)",
                (long long)stride_block, (long long)stride_tok);
  if (!aligned16(q_bd) || !aligned16(cos_sin) || !aligned16(rope_blocks))
    return fail(BELT_ERR_INVALID, "latent_decode: q_bd, cos_sin and rope_blocks must be 16-byte aligned");
  if (part_sh < lv + 1 || part_ss < 24 * part_sh) return fail(BELT_ERR_INVALID, "latent_decode: part strides");
  if (max_pos < 1) return fail(BELT_ERR_INVALID, "latent_decode: max_pos %d", max_pos);

  DecodeParams p{};
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.work = work;
  p.cta_seg = cta_seg;
  p.rope_blocks = static_cast<const __nv_bfloat16*>(rope_blocks);
  p.rope_ld = n_rope_blocks * 64;
  p.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin);
  p.max_pos = max_pos;
  p.part = part;
  p.part_ss = part_ss;
  p.part_sh = part_sh;
  p.err = err;
  p.cta_ns = reinterpret_cast<unsigned long long*>(cta_ns);
  p.num_reqs = num_reqs;
  p.num_blocks = static_cast<int>(num_blocks);
  p.page = page;
  p.n_k = n_k;
  p.v_offset = lk_pad;
  p.r_v = lv;
  p.n_vc = (lv + 63) / 64;
  p.n_vp = (lv + 127) / 128;
  // chunked layout: 64-column-aligned parts and whole 64-column chunks inside every row slot
  const int row_chunks = (row_width + 63) / 64;
  const bool chunked = lk_pad % 64 == 0 && page % 8 == 0 && static_cast<int64_t>(row_chunks) * 64 <= stride_tok;
  p.chunked = chunked ? 1 : 0;
  if (chunked) {
    p.cps = 4;
    p.chunk_stride = 1024;
    p.atom_stride = 4096;
    p.v_chunk0 = lk_pad / 64;
  } else {
    p.cps = 2;
    p.chunk_stride = 16384;
    p.atom_stride = 1024;
    p.v_chunk0 = 0;
  }
  p.stage_bytes = p.cps * 128 * 128;
  p.n_ks = (n_k + p.cps - 1) / p.cps;
  p.n_vs = (p.n_vc + p.cps - 1) / p.cps;
  // rows per TMA box: a whole page up to 128 rows (chunked boxes stack 8-row groups, page boxes are plain rows)
  p.box_rows = page < 128 ? page : 128;
  p.n_pieces = 128 / p.box_rows;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  // rebuild K-steps: 16-column steps covering every group's [off, off + rr), read from its rope blocks; sorted by
  // column so that the steps of every key pair stage (128 columns) form one range
  struct Kstep { int col, src, group; };
  Kstep ks_list[kDecodeMaxKsteps];
  int nb_first = 0, nk = 0;
  for (int g = 0; g < kG; ++g) {
    const int off = rope_groups[2 * g], rr = rope_groups[2 * g + 1];
    if (rr <= 0 || rr > kRot || off < 0 || off + rr > lk_pad)
      return fail(BELT_ERR_INVALID, "latent_decode: rope group %d (%d, %d) outside the K part", g, off, rr);
    const int c_lo = off / 64, c_hi = (off + rr - 1) / 64;
    for (int ks = off / 16; ks <= (off + rr - 1) / 16; ++ks) {
      if (nk >= kDecodeMaxKsteps) return fail(BELT_ERR_INVALID, "latent_decode: too many rebuild K-steps");
      const int col = 16 * ks;
      ks_list[nk++] = Kstep{col, (nb_first + (col / 64 - c_lo)) * 64 + col % 64, g};
    }
    nb_first += c_hi - c_lo + 1;
  }
  if (nb_first != n_rope_blocks)
    return fail(BELT_ERR_INVALID, "latent_decode: %d rope blocks given, the groups need %d", n_rope_blocks, nb_first);
  for (int i = 1; i < nk; ++i)   // insertion sort by column (stable: a group's steps keep their order)
    for (int j = i; j > 0 && ks_list[j - 1].col > ks_list[j].col; --j) {
      const Kstep t = ks_list[j];
      ks_list[j] = ks_list[j - 1];
      ks_list[j - 1] = t;
    }
  for (int g = 0; g < kG; ++g) {
    const int off = rope_groups[2 * g], rr = rope_groups[2 * g + 1];
    p.rope_ks0[g] = off / 16;
    p.rope_ks1[g] = (off + rr - 1) / 16;
    p.rope_e0[g] = -1;
    for (int e = 0; e < nk; ++e)
      if (ks_list[e].group == g && ks_list[e].col == 16 * p.rope_ks0[g]) p.rope_e0[g] = e;
    for (int j = 0; j <= p.rope_ks1[g] - p.rope_ks0[g]; ++j) {
      const int e = p.rope_e0[g] + j;
      if (p.rope_e0[g] < 0 || e >= nk || ks_list[e].group != g || ks_list[e].col != 16 * (p.rope_ks0[g] + j))
        return fail(BELT_ERR_INVALID, "latent_decode: RoPE coordinates of group %d interleave with another group's", g);
    }
  }
  // rebuild steps by key chunk: step ks = 4 cc + s of group g (ks0 <= ks <= ks1) reads image rope_e0[g] + ks - ks0
  for (int cc = 0; cc < n_k; ++cc) {
    unsigned long long v[2] = {0, 0};
    for (int s16 = 0; s16 < 4; ++s16) {
      const int ks = 4 * cc + s16;
      int w = 0;
      for (int g = 0; g < kG; ++g)
        if (ks >= p.rope_ks0[g] && ks <= p.rope_ks1[g]) {
          if (w == 2)
            return fail(BELT_ERR_INVALID, "latent_decode: columns %d-%d hold RoPE coordinates of three groups", 16 * ks,
                        16 * ks + 15);
          const unsigned f = 0x8000u | (ks != p.rope_ks0[g] ? 0x4000u : 0u) |
                             (static_cast<unsigned>(p.rope_e0[g] + ks - p.rope_ks0[g]) << 2) | static_cast<unsigned>(g);
          v[w++] |= static_cast<unsigned long long>(f) << (16 * s16);
        }
    }
    p.k_rebuild[cc][0] = v[0];
    p.k_rebuild[cc][1] = v[1];
    // as runs: the chunk's rebuild steps as at most two runs of consecutive steps of one group with consecutive
    // images; word 1 = bit 63 | run 0 | run 1 << 16, a run = bit 15 | step 0's accumulate flag << 14 | first image << 6
    // | group << 4 | (count - 1) << 2 | first step. The issuer then emits each run without per-step tests.
    struct Run { int step, count, group, image, acc; };
    Run runs[8];
    int n_runs = 0;
    bool fits = true;
    for (int s16 = 0; s16 < 4; ++s16)
      for (int w = 0; w < 2; ++w) {
        const unsigned f = static_cast<unsigned>(v[w] >> (16 * s16)) & 0xFFFFu;
        if (!(f & 0x8000u)) continue;
        const int g = static_cast<int>(f & 3u), e = static_cast<int>((f >> 2) & 63u), acc = (f >> 14) & 1u;
        bool joined = false;
        for (int r = 0; r < n_runs && !joined; ++r)
          if (runs[r].group == g && runs[r].step + runs[r].count == s16 && runs[r].image + runs[r].count == e && acc) {
            ++runs[r].count;
            joined = true;
          }
        if (!joined) {
          if (n_runs == 8) fits = false;
          else runs[n_runs++] = Run{s16, 1, g, e, static_cast<int>(acc)};
        }
      }
    if (fits && n_runs <= 2) {   // no run at all (a chunk without RoPE coordinates): bit 63 alone
      unsigned long long word = 1ull << 63;
      for (int r = 0; r < n_runs; ++r)
        word |= static_cast<unsigned long long>(0x8000u | (static_cast<unsigned>(runs[r].acc) << 14) |
                                                (static_cast<unsigned>(runs[r].image) << 6) |
                                                (static_cast<unsigned>(runs[r].group) << 4) |
                                                (static_cast<unsigned>(runs[r].count - 1) << 2) |
                                                static_cast<unsigned>(runs[r].step))
                << (16 * r);
      p.k_rebuild[cc][1] = word;
    }
  }
  for (int e = 0; e < nk; ++e) p.kst_src[e] = ks_list[e].src;   // the rotation warps build image e from these columns
  p.n_kst = nk;
  bool planned = decode_plan_smem(p);
  if (!planned && chunked) {   // two 64 KB stages do not fit next to this query / rebuild layout: 32 KB page stages
    p.chunked = 0;
    p.cps = 2;
    p.chunk_stride = 16384;
    p.atom_stride = 1024;
    p.v_chunk0 = 0;
    p.stage_bytes = p.cps * 128 * 128;
    p.n_ks = (n_k + p.cps - 1) / p.cps;
    p.n_vs = (p.n_vc + p.cps - 1) / p.cps;
    planned = decode_plan_smem(p);
  }
  if (!planned)
    return fail(BELT_ERR_INVALID, "latent_decode: layout (n_k %d, %d rebuild steps) does not fit in shared memory", n_k, nk);
  if (!decode_plan_stages(p))
    return fail(BELT_ERR_INVALID, "latent_decode: %d key and %d value chunks need more than %d ring stages", n_k, p.n_vc,
                kDecodeMaxPlan);
  const bool use_chunked = p.chunked != 0;

  DecodeMaps maps;
  if (use_chunked) {
    // {64 columns, 8 rows, 64-column chunks, 8-row groups of a page, blocks}; box {64, 8, n, box_rows / 8, 1} for
    // n = 1..4 chunks: the chunk index sits between the rows of a group and the groups, so each 8-row group of the box
    // lands as one n-chunk atom in shared memory
    cuuint64_t dims[5] = {64, 8, static_cast<cuuint64_t>(row_chunks), static_cast<cuuint64_t>(page / 8),
                          static_cast<cuuint64_t>(num_blocks)};
    cuuint64_t strides[4] = {static_cast<cuuint64_t>(stride_tok) * 2, 128, static_cast<cuuint64_t>(stride_tok) * 16,
                             static_cast<cuuint64_t>(stride_block) * 2};
    for (int n = 1; n <= 4; ++n) {
      cuuint32_t box[5] = {64, 8, static_cast<cuuint32_t>(n), static_cast<cuuint32_t>(p.box_rows / 8), 1};
      int r = encode_bf16(&maps.cache[n - 1], cache, 5, dims, strides, box, "cache");
      if (r != BELT_OK) return r;
    }
  } else {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(row_width), static_cast<cuuint64_t>(page),
                          static_cast<cuuint64_t>(num_blocks)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_tok) * 2, static_cast<cuuint64_t>(stride_block) * 2};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(p.box_rows), 1};
    int r = encode_bf16(&maps.cache[0], cache, 3, dims, strides, box, "cache");
    if (r != BELT_OK) return r;
    for (int n = 1; n < 4; ++n) maps.cache[n] = maps.cache[0];
  }
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kq), static_cast<cuuint64_t>(num_reqs) * kH};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kq) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kH)};
    int r = encode_bf16(&maps.q, q_bd, 2, dims, strides, box, "q_bd");
    if (r != BELT_OK) return r;
  }
  cudaError_t e = launch_latent_decode(maps, p, num_ctas, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "latent_decode launch");
}
}  // namespace

int belt_latent_decode(const void* q_bd, int32_t num_reqs, int32_t kq, const void* cache, int64_t num_blocks,
                       int32_t page, int32_t row_width, int64_t stride_block, int64_t stride_tok,
                       const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens, const int32_t* work,
                       const int32_t* cta_seg, int32_t num_ctas, float* part, int64_t part_ss, int64_t part_sh,
                       float sm_scale, int32_t lk_pad, int32_t lv, const int32_t* rope_groups,
                       const void* rope_blocks, int32_t n_rope_blocks, const void* cos_sin, int32_t max_pos,
                       int32_t* err, void* stream) {
  return latent_decode_impl(q_bd, num_reqs, kq, cache, num_blocks, page, row_width, stride_block, stride_tok,
                            block_table, bt_stride, seq_lens, work, cta_seg, num_ctas, part, part_ss, part_sh, sm_scale,
                            lk_pad, lv, rope_groups, rope_blocks, n_rope_blocks, cos_sin, max_pos, err, nullptr, stream);
}

int belt_latent_decode_timed(const void* q_bd, int32_t num_reqs, int32_t kq, const void* cache, int64_t num_blocks,
                             int32_t page, int32_t row_width, int64_t stride_block, int64_t stride_tok,
                             const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                             const int32_t* work, const int32_t* cta_seg, int32_t num_ctas, float* part,
                             int64_t part_ss, int64_t part_sh, float sm_scale, int32_t lk_pad, int32_t lv,
                             const int32_t* rope_groups, const void* rope_blocks, int32_t n_rope_blocks,
                             const void* cos_sin, int32_t max_pos, int32_t* err, int64_t* cta_ns, void* stream) {
  if (!cta_ns) return fail(BELT_ERR_INVALID, "latent_decode_timed: null cta_ns");
  return latent_decode_impl(q_bd, num_reqs, kq, cache, num_blocks, page, row_width, stride_block, stride_tok,
                            block_table, bt_stride, seq_lens, work, cta_seg, num_ctas, part, part_ss, part_sh, sm_scale,
                            lk_pad, lv, rope_groups, rope_blocks, n_rope_blocks, cos_sin, max_pos, err, cta_ns, stream);
}

}  // extern "C"

namespace {

// The piece list of a varlen decompress: host [n][4] = (request row of block_table, seq_len, pos0, count); outputs
// concatenated in piece order. Runs ceil(n / kVarlenMax) launches.
int decompress_pieces(const char* who, const void* cache, int64_t num_blocks, int32_t page, int32_t row_width,
                      int64_t stride_block, int64_t stride_tok, const int32_t* block_table, int64_t bt_stride,
                      int32_t num_pieces, const int32_t* pieces, const void* wk, int32_t kc, const int32_t* k_segs,
                      const void* v_up, int32_t v_offset, int32_t r_v, const void* cos_sin, int32_t max_pos,
                      void* k_out, void* v_out, int64_t out_st, int64_t out_sg, int32_t* err, cudaStream_t stream) {
  using namespace belt;
  if (num_pieces < 0 || (num_pieces > 0 && !pieces)) return fail(BELT_ERR_INVALID, "%s: piece list", who);
  long long total = 0;
  for (int i = 0; i < num_pieces; ++i) {
    const int req = pieces[4 * i], seq_len = pieces[4 * i + 1], pos0 = pieces[4 * i + 2], count = pieces[4 * i + 3];
    if (req < 0 || count < 0 || pos0 < 0 || seq_len < 0 || static_cast<int64_t>(pos0) + count > seq_len)
      return fail(BELT_ERR_INVALID, "%s: piece %d: positions [%d, %d) outside the request's %d (request %d)", who, i,
                  pos0, pos0 + count, seq_len, req);
    if (seq_len > max_pos)
      return fail(BELT_ERR_INVALID, "%s: cos_sin has %d rows < %d", who, max_pos, seq_len);
    total += count;
  }
  if (total == 0) return ok();
  if (!cache || !block_table || !wk || !k_segs || !v_up || !cos_sin || !k_out || !v_out)
    return fail(BELT_ERR_INVALID, "%s: null buffer", who);
  if (!(page == 16 || page == 32 || page == 64 || (page % 128 == 0 && page > 0)))
    return fail(BELT_ERR_INVALID, "%s: page size %d (supported: 16, 32, 64 or a multiple of 128)", who, page);
  if (num_blocks < 1 || num_blocks > (1ll << 31) - 2 || row_width <= 0 || stride_tok < row_width || stride_tok % 8 ||
      stride_block % 8 || !aligned16(cache))
    return fail(BELT_ERR_INVALID, "%s: cache rows must be 16-byte aligned (strides %lld, %lld)", who,
                (long long)stride_block, (long long)stride_tok);
  if (kc <= 0 || kc % 64 || kc > row_width + 63 || r_v <= 0 || r_v > 1024 || v_offset < 0 || v_offset + r_v > row_width)
    return fail(BELT_ERR_INVALID, "%s: kc %d, v_offset %d, r_v %d, row width %d", who, kc, v_offset, r_v, row_width);
  if (!aligned16(wk) || !aligned16(v_up) || !aligned16(k_out) || !aligned16(v_out) || out_st % 8 || out_sg % 8 ||
      out_sg < 256 || out_st < 4 * out_sg)
    return fail(BELT_ERR_INVALID, "%s: weights and outputs 16-byte aligned, output strides", who);
  DecompressParams p{};
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.page = page;
  p.num_blocks = static_cast<int>(num_blocks);
  for (int g = 0; g < kG; ++g) {
    const int runs[2][2] = {{k_segs[4 * g], k_segs[4 * g + 1]}, {k_segs[4 * g + 2], k_segs[4 * g + 3]}};
    bool use[64] = {};
    for (int q = 0; q < 2; ++q) {
      if (runs[q][1] <= 0) continue;
      if (runs[q][0] < 0 || runs[q][0] + runs[q][1] > kc)
        return fail(BELT_ERR_INVALID, "%s: k_segs of group %d outside the key part", who, g);
      for (int c = runs[q][0] >> 6; c <= (runs[q][0] + runs[q][1] - 1) >> 6 && c < 64; ++c) use[c] = true;
    }
    int n = 0;
    for (int c = 0; c < 64; ++c)
      if (use[c]) {
        if (n == kPwMaxChunks)
          return fail(BELT_ERR_INVALID, "%s: group %d spans more than %d 64-column chunks", who, g, kPwMaxChunks);
        p.k_chunk[g][n++] = c;
      }
    p.k_nch[g] = n;
  }
  p.v_offset = v_offset;
  p.v_chunk0 = v_offset / 64;
  p.v_nch = (v_offset + r_v + 63) / 64 - p.v_chunk0;
  p.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin);
  p.max_pos = max_pos;
  p.k_out = static_cast<__nv_bfloat16*>(k_out);
  p.v_out = static_cast<__nv_bfloat16*>(v_out);
  p.out_st = out_st;
  p.out_sg = out_sg;
  p.err = err;
  DecompressMaps maps;
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(row_width), static_cast<cuuint64_t>(page),
                          static_cast<cuuint64_t>(num_blocks)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_tok) * 2, static_cast<cuuint64_t>(stride_block) * 2};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(page < 128 ? page : 128), 1};
    int r = encode_bf16(&maps.cache, cache, 3, dims, strides, box, "cache");
    if (r != BELT_OK) return r;
  }
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kc), 256, static_cast<cuuint64_t>(kG)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(kc) * 2, static_cast<cuuint64_t>(kc) * 256 * 2};
    cuuint32_t box[3] = {64, 256, 1};
    int r = encode_bf16(&maps.wk, wk, 3, dims, strides, box, "wk");
    if (r != BELT_OK) return r;
  }
  {
    cuuint64_t dims[3] = {256, static_cast<cuuint64_t>(r_v), static_cast<cuuint64_t>(kG)};
    cuuint64_t strides[2] = {256 * 2, static_cast<cuuint64_t>(r_v) * 256 * 2};
    cuuint32_t box[3] = {64, 64, 1};
    int r = encode_bf16(&maps.v, v_up, 3, dims, strides, box, "v_up");
    if (r != BELT_OK) return r;
  }
  long long row = 0;
  for (int i0 = 0; i0 < num_pieces; i0 += kVarlenMax) {
    const int n = num_pieces - i0 < kVarlenMax ? num_pieces - i0 : kVarlenMax;
    p.num_pieces = n;
    p.piece_cta0[0] = 0;
    for (int i = 0; i < n; ++i) {
      const int* pc = pieces + 4 * (i0 + i);
      p.piece_req[i] = pc[0];
      p.piece_len[i] = pc[1];
      p.piece_pos0[i] = pc[2];
      p.piece_count[i] = pc[3];
      p.piece_out[i] = row;
      row += pc[3];
      p.piece_cta0[i + 1] = p.piece_cta0[i] + decompress_piece_ctas(pc[2], pc[3]);
    }
    cudaError_t e = launch_decompress(maps, p, stream);
    if (e != cudaSuccess) return cuda_fail(e, "latent_decompress launch");
  }
  return ok();
}

// The piece list of a varlen prefill attention: host [n][8] = (q_row, ql, k_row, S, q_pos0, k_pos0, o_row, to2).
int prefill_pieces(const char* who, const void* q, int64_t q_rows, int64_t q_st, int64_t q_sh, const void* k,
                   const void* v, int64_t k_rows, int64_t kv_st, int64_t kv_sg, int32_t num_pieces,
                   const int32_t* pieces, int32_t causal, float scale, void* out, void* out2, int64_t out_st,
                   int64_t out_sh, float* lse, float* lse2, int64_t lse_st, int32_t* err, cudaStream_t stream) {
  using namespace belt;
  if (num_pieces < 0 || (num_pieces > 0 && !pieces) || q_rows < 0 || k_rows < 0)
    return fail(BELT_ERR_INVALID, "%s: piece list", who);
  long long tiles = 0;
  bool any_keys = false;
  for (int i = 0; i < num_pieces; ++i) {
    const int* pc = pieces + 8 * i;
    if (pc[1] < 0 || pc[3] < 0 || pc[0] < 0 || pc[2] < 0 || pc[6] < 0 || pc[0] + static_cast<int64_t>(pc[1]) > q_rows ||
        pc[2] + static_cast<int64_t>(pc[3]) > k_rows)
      return fail(BELT_ERR_INVALID, "%s: piece %d: query rows [%d, +%d) of %lld, key rows [%d, +%d) of %lld", who, i,
                  pc[0], pc[1], (long long)q_rows, pc[2], pc[3], (long long)k_rows);
    if (pc[7] && !out2) return fail(BELT_ERR_INVALID, "%s: piece %d writes to out2, which is null", who, i);
    tiles += (pc[1] + 127) / 128;
    any_keys = any_keys || pc[3] > 0;
  }
  if (tiles == 0) return ok();
  if (!q || !out || (any_keys && (!k || !v))) return fail(BELT_ERR_INVALID, "%s: null buffer", who);
  if (!aligned16(q) || !aligned16(out) || (out2 && !aligned16(out2)) || (any_keys && (!aligned16(k) || !aligned16(v))) ||
      q_st % 8 || q_sh % 8 || kv_st % 8 || kv_sg % 8 || out_st % 8 || out_sh % 8 || q_sh < 256 || q_st < kH * q_sh ||
      kv_sg < 256 || kv_st < kG * kv_sg || out_sh < 256 || out_st < kH * out_sh)
    return fail(BELT_ERR_INVALID, "%s: 16-byte aligned tensors, strides multiples of 8 elements", who);
  if ((lse || lse2) && lse_st < kH) return fail(BELT_ERR_INVALID, "%s: lse row stride %lld", who, (long long)lse_st);
  PrefillAttnParams p{};
  p.H = kH;
  p.hpg = kHPG;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out2 = static_cast<__nv_bfloat16*>(out2);
  p.out_st = out_st;
  p.out_sh = out_sh;
  p.lse = lse;
  p.lse2 = lse2;
  p.lse_st = lse_st;
  p.err = err;
  PrefillAttnMaps maps;
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(kH), static_cast<cuuint64_t>(q_rows)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(q_sh) * 2, static_cast<cuuint64_t>(q_st) * 2};
    cuuint32_t box[3] = {64, 1, 128};
    int r = encode_bf16(&maps.q, q, 3, dims, strides, box, "q");
    if (r != BELT_OK) return r;
  }
  const long long nk = k_rows > 0 ? k_rows : 1;   // a map of one row when there are no keys (never read)
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(kG), static_cast<cuuint64_t>(nk)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(kv_sg) * 2, static_cast<cuuint64_t>(kv_st) * 2};
    cuuint32_t box[3] = {64, 1, 128};
    int r = encode_bf16(&maps.k, any_keys ? k : q, 3, dims, strides, box, "k");
    if (r != BELT_OK) return r;
    r = encode_bf16(&maps.v, any_keys ? v : q, 3, dims, strides, box, "v");
    if (r != BELT_OK) return r;
  }
  for (int i0 = 0; i0 < num_pieces; i0 += kVarlenMax) {
    const int n = num_pieces - i0 < kVarlenMax ? num_pieces - i0 : kVarlenMax;
    p.num_pieces = n;
    p.piece_cta0[0] = 0;
    for (int i = 0; i < n; ++i) {
      const int* pc = pieces + 8 * (i0 + i);
      p.piece_q_row[i] = pc[0];
      p.piece_ql[i] = pc[1];
      p.piece_k_row[i] = pc[2];
      p.piece_S[i] = pc[3];
      p.piece_q_pos0[i] = pc[4];
      p.piece_k_pos0[i] = pc[5];
      p.piece_o_row[i] = pc[6];
      p.piece_to2[i] = pc[7];
      p.piece_cta0[i + 1] = p.piece_cta0[i] + (pc[1] + 127) / 128;
    }
    cudaError_t e = launch_prefill_attn(maps, p, stream);
    if (e != cudaSuccess) return cuda_fail(e, "prefill_attention launch");
  }
  return ok();
}

}  // namespace

extern "C" {

int belt_latent_decompress(const void* cache, int64_t num_blocks, int32_t page, int32_t row_width,
                           int64_t stride_block, int64_t stride_tok, const int32_t* block_table_row, int32_t seq_len,
                           int32_t pos0, int32_t count, const void* wk, int32_t kc, const int32_t* k_segs,
                           const void* v_up, int32_t v_offset, int32_t r_v, const void* cos_sin, int32_t max_pos,
                           void* k_out, void* v_out, int64_t out_st, int64_t out_sg, int32_t* err, void* stream) {
  const int32_t piece[4] = {0, seq_len, pos0, count};
  return decompress_pieces("latent_decompress", cache, num_blocks, page, row_width, stride_block, stride_tok,
                           block_table_row, 0, 1, piece, wk, kc, k_segs, v_up, v_offset, r_v, cos_sin, max_pos, k_out,
                           v_out, out_st, out_sg, err, as_stream(stream));
}

int belt_latent_decompress_varlen(const void* cache, int64_t num_blocks, int32_t page, int32_t row_width,
                                  int64_t stride_block, int64_t stride_tok, const int32_t* block_table,
                                  int64_t bt_stride, int32_t num_pieces, const int32_t* pieces, const void* wk,
                                  int32_t kc, const int32_t* k_segs, const void* v_up, int32_t v_offset, int32_t r_v,
                                  const void* cos_sin, int32_t max_pos, void* k_out, void* v_out, int64_t out_st,
                                  int64_t out_sg, int32_t* err, void* stream) {
  return decompress_pieces("latent_decompress_varlen", cache, num_blocks, page, row_width, stride_block, stride_tok,
                           block_table, bt_stride, num_pieces, pieces, wk, kc, k_segs, v_up, v_offset, r_v, cos_sin,
                           max_pos, k_out, v_out, out_st, out_sg, err, as_stream(stream));
}

int belt_prefill_attention(const void* q, int32_t ql, int64_t q_st, int64_t q_sh, const void* k, const void* v,
                           int32_t num_keys, int64_t kv_st, int64_t kv_sg, int32_t q_pos0, int32_t k_pos0,
                           int32_t causal, float scale, void* out, int64_t out_st, int64_t out_sh, float* lse,
                           int64_t lse_st, int32_t* err, void* stream) {
  if (ql < 0 || num_keys < 0) return fail(BELT_ERR_INVALID, "prefill_attention: ql %d, keys %d", ql, num_keys);
  const int32_t piece[8] = {0, ql, 0, num_keys, q_pos0, k_pos0, 0, 0};
  return prefill_pieces("prefill_attention", q, ql, q_st, q_sh, k, v, num_keys, kv_st, kv_sg, 1, piece, causal, scale,
                        out, nullptr, out_st, out_sh, lse, nullptr, lse_st, err, as_stream(stream));
}

int belt_prefill_attention_varlen(const void* q, int64_t q_rows, int64_t q_st, int64_t q_sh, const void* k,
                                  const void* v, int64_t k_rows, int64_t kv_st, int64_t kv_sg, int32_t num_pieces,
                                  const int32_t* pieces, int32_t causal, float scale, void* out, void* out2,
                                  int64_t out_st, int64_t out_sh, float* lse, float* lse2, int64_t lse_st,
                                  int32_t* err, void* stream) {
  return prefill_pieces("prefill_attention_varlen", q, q_rows, q_st, q_sh, k, v, k_rows, kv_st, kv_sg, num_pieces,
                        pieces, causal, scale, out, out2, out_st, out_sh, lse, lse2, lse_st, err, as_stream(stream));
}

int belt_attn_fold(void* out, int64_t out_st, int64_t out_sh, float* lse, int64_t lse_st, const void* part,
                   int64_t part_st, int64_t part_sh, const float* part_lse, int64_t plse_st, int32_t num_pieces,
                   const int32_t* pieces, void* stream) {
  using namespace belt;
  if (num_pieces < 0 || (num_pieces > 0 && !pieces)) return fail(BELT_ERR_INVALID, "attn_fold: piece list");
  long long rows = 0;
  for (int i = 0; i < num_pieces; ++i) {
    if (pieces[3 * i] < 0 || pieces[3 * i + 1] < 0 || pieces[3 * i + 2] < 0)
      return fail(BELT_ERR_INVALID, "attn_fold: piece %d", i);
    rows += pieces[3 * i + 2];
  }
  if (rows == 0) return ok();
  if (!out || !lse || !part || !part_lse) return fail(BELT_ERR_INVALID, "attn_fold: null buffer");
  if (!aligned16(out) || !aligned16(part) || out_st % 8 || out_sh % 8 || part_st % 8 || part_sh % 8 || out_sh < 256 ||
      part_sh < 256 || lse_st < kH || plse_st < kH)
    return fail(BELT_ERR_INVALID, "attn_fold: 16-byte aligned rows, strides multiples of 8 elements");
  AttnFoldParams p{};
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_st = out_st;
  p.out_sh = out_sh;
  p.lse = lse;
  p.lse_st = lse_st;
  p.part = static_cast<const __nv_bfloat16*>(part);
  p.part_st = part_st;
  p.part_sh = part_sh;
  p.plse = part_lse;
  p.plse_st = plse_st;
  p.H = kH;
  for (int i0 = 0; i0 < num_pieces; i0 += kVarlenMax) {
    const int n = num_pieces - i0 < kVarlenMax ? num_pieces - i0 : kVarlenMax;
    p.num_pieces = n;
    p.piece_row0[0] = 0;
    for (int i = 0; i < n; ++i) {
      p.piece_dst[i] = pieces[3 * (i0 + i)];
      p.piece_src[i] = pieces[3 * (i0 + i) + 1];
      p.piece_rows[i] = pieces[3 * (i0 + i) + 2];
      p.piece_row0[i + 1] = p.piece_row0[i] + p.piece_rows[i];
    }
    cudaError_t e = launch_attn_fold(p, as_stream(stream));
    if (e != cudaSuccess) return cuda_fail(e, "attn_fold launch");
  }
  return ok();
}

int belt_q_norm_rope(const void* qg, int32_t num_tokens, int64_t qg_st, int64_t qg_sh, const float* norm_weight,
                     float eps, const void* cos_sin, int32_t max_pos, int32_t rot, const void* positions,
                     int32_t positions_i64, void* q, int64_t q_st, int64_t q_sh, void* stream) {
  using namespace belt;
  if (num_tokens < 0 || rot < 16 || rot > 256 || rot % 16 || max_pos < 1 || eps < 0.f)
    return fail(BELT_ERR_INVALID, "q_norm_rope: tokens %d, rot %d (a multiple of 16 up to 256), max_pos %d", num_tokens,
                rot, max_pos);
  if (num_tokens == 0) return ok();
  if (!qg || !norm_weight || !cos_sin || !positions || !q) return fail(BELT_ERR_INVALID, "q_norm_rope: null buffer");
  if (!aligned16(qg) || !aligned16(q) || qg_st % 8 || qg_sh % 8 || q_st % 8 || q_sh % 8 || q_sh < 256 ||
      q_st < kH * q_sh)
    return fail(BELT_ERR_INVALID, "q_norm_rope: 16-byte aligned rows, strides multiples of 8 elements");
  QNormRopeParams p{static_cast<const __nv_bfloat16*>(qg), qg_st, qg_sh, num_tokens, kH, norm_weight, eps,
                    static_cast<const __nv_bfloat16*>(cos_sin), max_pos, rot, positions, positions_i64 ? 1 : 0,
                    static_cast<__nv_bfloat16*>(q), q_st, q_sh};
  cudaError_t e = launch_q_norm_rope(p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "q_norm_rope launch");
}

int belt_gate_mul(const void* attn, int64_t attn_st, int64_t attn_sh, const void* gate, int64_t gate_st,
                  int64_t gate_sh, int32_t num_tokens, void* out, int64_t out_st, int64_t out_sh, void* stream) {
  using namespace belt;
  if (num_tokens < 0) return fail(BELT_ERR_INVALID, "gate_mul: tokens %d", num_tokens);
  if (num_tokens == 0) return ok();
  if (!attn || !gate || !out) return fail(BELT_ERR_INVALID, "gate_mul: null buffer");
  if (!aligned16(attn) || !aligned16(gate) || !aligned16(out) || attn_st % 8 || attn_sh % 8 || gate_st % 8 ||
      gate_sh % 8 || out_st % 8 || out_sh % 8)
    return fail(BELT_ERR_INVALID, "gate_mul: 16-byte aligned rows, strides multiples of 8 elements");
  GateMulParams p{static_cast<const __nv_bfloat16*>(attn), attn_st, attn_sh, static_cast<const __nv_bfloat16*>(gate),
                  gate_st, gate_sh, num_tokens, kH, static_cast<__nv_bfloat16*>(out), out_st, out_sh};
  cudaError_t e = launch_gate_mul(p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "gate_mul launch");
}

int belt_merge_up_project(const float* part, int64_t part_ss, int64_t part_sh, const int32_t* seg_base,
                          int32_t num_reqs, int32_t lv, const void* v_up_t, void* out, int64_t out_st, int64_t out_sh,
                          float* lse, int64_t lse_sb, int32_t* err, void* stream) {
  using namespace belt;
  if (num_reqs < 0 || lv <= 0 || lv > 640)
    return fail(BELT_ERR_INVALID, "merge_up_project: num_reqs %d, lv %d (at most 640)", num_reqs, lv);
  if (num_reqs == 0) return ok();
  if (!part || !seg_base || !v_up_t || !out) return fail(BELT_ERR_INVALID, "merge_up_project: null buffer");
  if (part_sh < lv + 1 || part_ss < kH * part_sh || !aligned16(v_up_t) || (lse && lse_sb < kH))
    return fail(BELT_ERR_INVALID, "merge_up_project: part strides, v_up_t alignment or lse stride");
  MergeUpParams p{part, part_ss, part_sh, seg_base, num_reqs, kH, kHPG, lv, static_cast<__nv_bfloat16*>(out),
                  out_st, out_sh, lse, lse_sb, err};
  p.vec_part = aligned16(part) && part_ss % 4 == 0 && part_sh % 4 == 0 && lv % 4 == 0;
  p.vec_out = aligned16(out) && out_st % 8 == 0 && out_sh % 8 == 0;
  MergeUpMaps maps;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(lv), static_cast<cuuint64_t>(kG)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(lv) * kD * 2};
  cuuint32_t box[3] = {64, 64, 1};
  int r = encode_bf16(&maps.v, v_up_t, 3, dims, strides, box, "v_up_t");
  if (r != BELT_OK) return r;
  cudaError_t e = launch_merge_up(maps, p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "merge_up_project launch");
}

int belt_gemm_bf16(const void* a, int64_t m, int64_t k, int64_t lda, const void* b, int64_t n, int64_t ldb, void* c,
                   int64_t ldc, int32_t* err, void* stream) {
  using namespace belt;
  if (m < 0 || n < 0 || k <= 0 || m > (1ll << 31) - 1 || n > (1ll << 31) - 1 || k > (1ll << 31) - 1)
    return fail(BELT_ERR_INVALID, "gemm_bf16: m %lld, n %lld, k %lld", (long long)m, (long long)n, (long long)k);
  if (m == 0 || n == 0) return ok();
  if (!a || !b || !c) return fail(BELT_ERR_INVALID, "gemm_bf16: null buffer");
  if (k % 8 || lda < k || ldb < k || lda % 8 || ldb % 8 || ldc < n || !aligned16(a) || !aligned16(b))
    return fail(BELT_ERR_INVALID, "gemm_bf16: k %lld and the row strides (%lld, %lld) must be multiples of 8, a and b "
                "16-byte aligned", (long long)k, (long long)lda, (long long)ldb);
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  GemmParams p{};
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.tiles_m = static_cast<int>((m + 127) / 128);
  // 256-column tiles when they still give every SM a tile, 128 otherwise (more, smaller tiles for small products)
  const long long tiles256 = p.tiles_m * ((n + 255) / 256);
  p.bn = tiles256 >= sms ? 256 : 128;
  p.num_tiles = static_cast<int>(p.tiles_m * ((n + p.bn - 1) / p.bn));
  p.vec_out = aligned16(c) && ldc % 8 == 0;
  p.err = err;
  GemmMaps maps;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(lda) * 2};
    cuuint32_t box[2] = {64, 128};
    int r = encode_bf16(&maps.a, a, 2, dims, strides, box, "gemm a");
    if (r != BELT_OK) return r;
  }
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(n)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldb) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(p.bn)};
    int r = encode_bf16(&maps.b, b, 2, dims, strides, box, "gemm b");
    if (r != BELT_OK) return r;
  }
  cudaError_t e = launch_gemm(maps, p, sms, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "gemm_bf16 launch");
}

int belt_selftest_bounded_wait(int32_t* err, int32_t* status, void* stream) {
  if (!err || !status) return fail(BELT_ERR_INVALID, "selftest_bounded_wait: null buffer");
  cudaError_t e = belt::launch_selftest_wait(err, status, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "selftest_bounded_wait launch");
}

int belt_merge_segments(const float* part, int64_t part_ss, int64_t part_sh, const int32_t* seg_base,
                        int32_t num_reqs, int32_t nh, int32_t lv, void* out, int64_t out_sb, int64_t out_sh,
                        float* lse, int64_t lse_sb, void* stream) {
  if (num_reqs < 0 || nh <= 0 || lv <= 0 || lv > 1024) return fail(BELT_ERR_INVALID, "merge_segments: bad arguments");
  if (num_reqs == 0) return ok();
  if (!part || !seg_base || !out || !lse) return fail(BELT_ERR_INVALID, "merge_segments: null buffer");
  belt::MergeParams p{part, part_ss, part_sh, seg_base, num_reqs, nh, lv, static_cast<__nv_bfloat16*>(out),
                      out_sb, out_sh, lse, lse_sb};
  cudaError_t e = belt::launch_merge(p, as_stream(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "merge_segments launch");
}

}  // extern "C"
